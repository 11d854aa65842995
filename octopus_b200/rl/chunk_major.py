"""Chunk-major training of one prefix-tree micro-batch: the tree runs through the whole
model one chunk of at most `tokens` tree rows at a time, so activation memory follows the
chunk, not the tree.

Chunks.  The micro-batch's attention sequences (tree nodes: query rows, key list =
mounted rows + ancestor path + own rows) are ordered topologically: a node after every node
owning one of its keys, otherwise by index (pre-order for a tree without mounts).  A node
longer than `tokens` is cut into parts; part [a, b) of a node attends to the node's key
list up to its row b (bottom-right causal).  Parts are packed into chunks of at most
`tokens` rows, in that order.

Kept tensors.  Per decoder layer, the k / v rows of every tree row that a later chunk's
queries read (an ancestor's, a mounted one, an earlier part of the query's own node) are
kept, one slot each, slots ordered by owning chunk: a chunk writes its own as one block
and reads earlier chunks' by index.  A chunk's attention keys are [its own rows ||
the kept rows it reads].  Hybrid models' linear-recurrence layers keep, the same way, the
final state of every part whose continuation (its node's next part, or a child node) runs
in a later chunk, and the conv input rows a later part's causal conv starts from
(_LinearPlan).

run_forward runs the chunks in order without autograd (keeping what later chunks read);
run_backward runs them in reverse with autograd: each layer is checkpointed, its inputs
being the layer input and the kept k / v it reads, so the recompute returns their
gradients, which are summed (fp32) into the owning chunk's slots; when that chunk runs,
the sums are the output gradients of the k / v it kept.  Parameter gradients add up to
those of the whole tree (they accumulate in the weights' main_grad buffers).
chunk_major_forward is both as one autograd op returning (logp, entropy) per scored pair.

Reference parity (behaviour): `octopus/rl/chunk_major.py:1-40` (chunk order, kept tensors,
reverse-chunk backward with gradient sums, one autograd op), `ChunkPlan` (`:73-168`),
`run_forward` / `run_backward` (`:326-363`), and for hybrid models the recurrent states and
convolution context rows kept across chunks.
"""
from __future__ import annotations

import heapq
from dataclasses import dataclass

import numpy as np
import torch

from .. import ops
from ..models.decoder import qkv_rope


@dataclass
class Chunk:
    rows: np.ndarray          # tree rows of the chunk's queries (its own rows), in chunk order
    n_pad: int                # rows incl. padding (a multiple of 8 for the GEMMs)
    ext_slots: np.ndarray     # kept slots of the earlier chunks' rows it reads (keys n_pad + j)
    own_lo: int               # its kept rows occupy slots [own_lo, own_hi) ...
    own_hi: int
    own_local: np.ndarray     # ... at these chunk rows
    cu_q: np.ndarray
    cu_k: np.ndarray
    key_local: np.ndarray     # keys as chunk rows (< n_pad) or n_pad + index into ext_slots
    pair_idx: np.ndarray      # micro-batch pair indices scored in this chunk
    pair_local: np.ndarray    # their chunk rows


class ChunkPlan:
    """The chunks of a micro-batch (rl.actor.MicroBatch) of at most `tokens` rows each."""

    def __init__(self, mb, tokens: int):
        tokens = max(8, int(tokens))
        cu_q, cu_k, key_idx = (np.asarray(a, np.int64) for a in (mb.cu_q, mb.cu_k, mb.key_idx))
        T = len(mb.tokens)
        nseq = len(cu_q) - 1
        row_seq = np.full(T, -1, np.int64)
        for s in range(nseq):
            row_seq[cu_q[s]:cu_q[s + 1]] = s
        keys = [key_idx[cu_k[s]:cu_k[s + 1]] for s in range(nseq)]
        order = _topological([set(np.unique(row_seq[k]).tolist()) - {s, -1} for s, k in enumerate(keys)])
        # parts (seq, a, b) of at most `tokens` query rows, packed into chunks
        chunk_parts, size = [[]], 0
        for s in order:
            nq = int(cu_q[s + 1] - cu_q[s])
            for a in range(0, nq, tokens):
                b = min(nq, a + tokens)
                if size + (b - a) > tokens and chunk_parts[-1]:
                    chunk_parts.append([])
                    size = 0
                chunk_parts[-1].append((s, a, b))
                size += b - a
        chunk_parts = [c for c in chunk_parts if c]
        row_chunk = np.full(T, -1, np.int64)
        row_local = np.full(T, -1, np.int64)
        rows_of = []
        for c, parts in enumerate(chunk_parts):
            rows = np.concatenate([np.arange(cu_q[s] + a, cu_q[s] + b) for s, a, b in parts])
            row_chunk[rows], row_local[rows] = c, np.arange(len(rows))
            rows_of.append(rows)
        # every key a chunk reads outside itself comes from an earlier chunk
        ext_of = []
        for c, parts in enumerate(chunk_parts):
            ks = np.concatenate([keys[s][: len(keys[s]) - (int(cu_q[s + 1] - cu_q[s]) - b)] for s, a, b in parts])
            e = np.unique(ks[row_chunk[ks] != c])
            assert (row_chunk[e] < c).all(), "chunk-major: a key row's chunk runs after its reader"
            ext_of.append(e)
        kept = np.unique(np.concatenate([np.empty(0, np.int64)] + ext_of))
        kept = kept[np.lexsort((row_local[kept], row_chunk[kept]))]  # slots by owning chunk, then row
        slot_of = np.full(T, -1, np.int64)
        slot_of[kept] = np.arange(len(kept))
        owner = row_chunk[kept]
        pair_row = np.asarray(mb.pair_row, np.int64)
        self.chunks: list[Chunk] = []
        for c, (parts, rows, e) in enumerate(zip(chunk_parts, rows_of, ext_of)):
            n = len(rows)
            n_pad = (n + 7) // 8 * 8
            e = e[np.argsort(slot_of[e])]
            ext_pos = np.full(T, -1, np.int64)
            ext_pos[e] = np.arange(len(e))
            cq, ck, kl = [0], [0], []
            q0 = 0
            for s, a, b in parts:
                ks = keys[s][: len(keys[s]) - (int(cu_q[s + 1] - cu_q[s]) - b)]
                kl.append(np.where(row_chunk[ks] == c, row_local[ks], n_pad + ext_pos[ks]))
                q0 += b - a
                cq.append(q0)
                ck.append(ck[-1] + len(ks))
            if n_pad > n:  # padding rows attend to themselves only
                kl.append(np.arange(n, n_pad))
                cq.append(n_pad)
                ck.append(ck[-1] + n_pad - n)
            lo, hi = (int(x) for x in np.searchsorted(owner, [c, c + 1]))
            pidx = np.flatnonzero(row_chunk[pair_row] == c)
            self.chunks.append(Chunk(rows, n_pad, slot_of[e], lo, hi, row_local[kept[lo:hi]],
                                     np.asarray(cq, np.int32), np.asarray(ck, np.int32),
                                     np.concatenate(kl).astype(np.int32), pidx, row_local[pair_row[pidx]]))
        self.n_kept = len(kept)
        self.n_pairs = len(pair_row)
        self.parts, self.cu_q = chunk_parts, cu_q
        self.row_chunk, self.row_local = row_chunk, row_local
        self.tokens = np.asarray(mb.tokens, np.int64)
        self.positions = np.asarray(mb.positions, np.int32)
        self.pair_label = np.asarray(mb.pair_label, np.int64)


def _topological(deps: list[set]) -> list[int]:
    """Indices ordered after their dependencies, the lowest ready index first."""
    users: list[list[int]] = [[] for _ in deps]
    for k, d in enumerate(deps):
        for j in d:
            users[j].append(k)
    waiting = [len(d) for d in deps]
    ready = [k for k, w in enumerate(waiting) if not w]
    heapq.heapify(ready)
    order = []
    while ready:
        k = heapq.heappop(ready)
        order.append(k)
        for u in users[k]:
            waiting[u] -= 1
            if not waiting[u]:
                heapq.heappush(ready, u)
    assert len(order) == len(deps), "chunk-major: key dependencies form a cycle"
    return order


class _DevChunk:
    """A chunk's tensors on the device."""

    def __init__(self, plan: ChunkPlan, ch: Chunk, device, c: int = 0):
        n, n_pad = len(ch.rows), ch.n_pad
        ids = np.zeros(n_pad, np.int64)
        pos = np.zeros(n_pad, np.int32)
        ids[:n], pos[:n] = plan.tokens[ch.rows], plan.positions[ch.rows]
        T = lambda a, dt: torch.as_tensor(np.ascontiguousarray(a), dtype=dt, device=device)  # noqa: E731
        self.ids, self.pos = T(ids, torch.int64), T(pos, torch.int32)
        self.plan = ops.AttnPlan.build(ch.cu_q, ch.cu_k, ch.key_local, device)
        self.ext = T(ch.ext_slots, torch.int64)
        self.own = T(ch.own_local, torch.int64)
        self.pair_idx = T(ch.pair_idx, torch.int64)
        self.pair_local = T(ch.pair_local, torch.int64)
        self.labels = T(plan.pair_label[ch.pair_idx], torch.int64)
        self.lo, self.hi = ch.own_lo, ch.own_hi
        lin = getattr(plan, "linear", None)
        self.lin = _DevLinear(lin.chunks[c], device) if lin is not None else None


class _LinearPlan:
    """Recurrent-layer bookkeeping of a ChunkPlan (hybrid models: rl uses models.hybrid).

    Units are the plan's parts (seq, a, b).  A unit's recurrence starts from the final
    state of its source: the previous part of its node (a > 0) or the last part of its
    parent node (a = 0; an empty parent passes its own parent's), zeros at the root.  A
    source in an earlier chunk is read from a kept state slot; one in the same chunk runs
    at an earlier level of that chunk.  A unit's causal conv starts from the W - 1 conv
    inputs before its first row on its ancestor path; those in earlier chunks are kept
    conv rows.  Slots are ordered by owning chunk, like the attention's kept rows."""

    def __init__(self, plan: ChunkPlan, mb, W: int):
        nodes, tails = np.asarray(mb.nodes, np.int64), np.asarray(mb.path_tail, np.int64)
        cu_q = plan.cu_q
        node_at = {int(nodes[k, 0]): k for k in range(len(nodes)) if nodes[k, 1] > nodes[k, 0]}
        seq_node = [node_at[int(cu_q[s])] for s in range(len(cu_q) - 1)]
        node_seq = {k: s for s, k in enumerate(seq_node)}
        units = []  # (chunk, seq, a, b, local offset)
        for c, parts in enumerate(plan.parts):
            off = 0
            for sq, a, b in parts:
                units.append((c, sq, a, b, off))
                off += b - a
        by_end = {(u[1], u[3]): j for j, u in enumerate(units)}
        src = []
        for c, sq, a, b, _ in units:
            if a > 0:
                src.append(by_end[(sq, a)])
                continue
            p = int(nodes[seq_node[sq], 2])
            while p >= 0 and nodes[p, 1] == nodes[p, 0]:
                p = int(nodes[p, 2])
            ps = node_seq.get(p) if p >= 0 else None
            src.append(by_end[(ps, int(cu_q[ps + 1] - cu_q[ps]))] if ps is not None else -1)
        chunk_of = np.asarray([u[0] for u in units], np.int64)
        st_units = sorted({v for j, v in enumerate(src) if v >= 0 and chunk_of[v] != chunk_of[j]},
                          key=lambda v: (chunk_of[v], v))
        st_slot = {v: j for j, v in enumerate(st_units)}
        rc, rl = plan.row_chunk, plan.row_local
        ctx_rows = []
        for c, sq, a, b, _ in units:
            k = seq_node[sq]
            path = [int(r) for r in tails[k] if r >= 0] + list(range(int(nodes[k, 0]), int(nodes[k, 0]) + a))
            path = path[-(W - 1):] if W > 1 else []
            ctx_rows.append([-1] * (W - 1 - len(path)) + path)
        cx_rows = sorted({r for j, rows in enumerate(ctx_rows) for r in rows if r >= 0 and rc[r] != chunk_of[j]},
                         key=lambda r: (rc[r], rl[r]))
        cx_slot = {r: j for j, r in enumerate(cx_rows)}
        self.n_state, self.n_conv = len(st_units), len(cx_rows)
        st_owner = np.asarray([chunk_of[v] for v in st_units], np.int64)
        cx_owner = np.asarray([rc[r] for r in cx_rows], np.int64)
        self.chunks = []
        for c, ch in enumerate(plan.chunks):
            mine = [j for j in range(len(units)) if chunk_of[j] == c]
            loc = {j: i for i, j in enumerate(mine)}
            n, n_pad = len(ch.rows), ch.n_pad
            segs = [(units[j][4], units[j][3] - units[j][2]) for j in mine]
            level = []
            for j in mine:
                v = src[j]
                level.append(level[loc[v]] + 1 if v >= 0 and chunk_of[v] == c else 0)
            if n_pad > n:  # the chunk's padding rows: one unit of its own
                segs.append((n, n_pad - n))
                level.append(0)
            ext_st = sorted({st_slot[src[j]] for j in mine if src[j] >= 0 and chunk_of[src[j]] != c})
            ext_st_pos = {sl: i for i, sl in enumerate(ext_st)}
            fin_pos, levels, nfin = {}, [], 0
            for lv in range(max(level) + 1 if level else 0):
                ids = [i for i, l_ in enumerate(level) if l_ == lv]
                init = []
                for i in ids:
                    j = mine[i] if i < len(mine) else -1
                    v = src[j] if j >= 0 else -1
                    if v < 0:
                        init.append(-1)
                    elif chunk_of[v] != c:
                        init.append(ext_st_pos[st_slot[v]])
                    else:
                        init.append(len(ext_st) + fin_pos[loc[v]])
                lens = [segs[i][1] for i in ids]
                rows = np.concatenate([np.arange(segs[i][0], segs[i][0] + segs[i][1]) for i in ids])
                starts = np.r_[0, np.cumsum(lens)[:-1]]
                levels.append((rows.astype(np.int64), list(zip(starts.tolist(), lens)), init))
                for i in ids:
                    fin_pos[i] = nfin
                    nfin += 1
            st_lo, st_hi = (int(x) for x in np.searchsorted(st_owner, [c, c + 1]))
            own_fin = [fin_pos[loc[v]] for v in st_units[st_lo:st_hi]]
            ext_cx = sorted({cx_slot[r] for j in mine for r in ctx_rows[j] if r >= 0 and rc[r] != c})
            ext_cx_pos = {sl: i for i, sl in enumerate(ext_cx)}
            cidx = [[int(rl[r]) if r >= 0 and rc[r] == c else (n_pad + ext_cx_pos[cx_slot[r]] if r >= 0 else -1)
                     for r in ctx_rows[j]] for j in mine]
            if n_pad > n:
                cidx.append([-1] * (W - 1))
            cx_lo, cx_hi = (int(x) for x in np.searchsorted(cx_owner, [c, c + 1]))
            self.chunks.append({"segs": segs, "levels": levels, "ext_state": np.asarray(ext_st, np.int64),
                                "ext_conv": np.asarray(ext_cx, np.int64),
                                "ctx_idx": np.asarray(cidx, np.int64).reshape(len(segs), W - 1),
                                "own_fin": np.asarray(own_fin, np.int64), "st": (st_lo, st_hi), "cx": (cx_lo, cx_hi),
                                "own_conv": np.asarray([rl[r] for r in cx_rows[cx_lo:cx_hi]], np.int64)})


class _DevLinear:
    def __init__(self, lc: dict, device):
        T = lambda a: torch.as_tensor(np.ascontiguousarray(a), dtype=torch.int64, device=device)  # noqa: E731
        self.segs = lc["segs"]
        self.levels = [(T(rows), segs, init) for rows, segs, init in lc["levels"]]
        self.ext_state, self.ext_conv = T(lc["ext_state"]), T(lc["ext_conv"])
        self.ctx_idx, self.own_fin, self.own_conv = T(lc["ctx_idx"]), T(lc["own_fin"]), T(lc["own_conv"])
        self.st, self.cx = lc["st"], lc["cx"]


def _chunk_linear_layer(x, st_ext, cx_ext, hw, i, L):
    """One linear-recurrence layer of a chunk (models.hybrid.linear_layer_forward on the
    chunk's units): initial states from kept states (st_ext) or earlier levels, conv context
    from chunk rows or kept conv rows (cx_ext); returns (layer output, the states and conv
    input rows it keeps for later chunks)."""
    from ..models.hybrid import _rmsnorm_heads
    from ..ops.recurrence import causal_conv, recurrence

    hc, cfg, t = hw.hc, hw.hc.base, hw.t
    h = ops.rmsnorm(x, t[f"layers.{i}.ln1"], cfg.rms_eps, cfg.norm_plus_one)
    qkv = ops.linear(h, t[f"layers.{i}.lin_qkv"])
    z = ops.linear(h, t[f"layers.{i}.lin_z"])
    ba = ops.linear(h, t[f"layers.{i}.lin_ba"])
    bb, aa = ba[:, :hc.lin_heads], ba[:, hc.lin_heads:2 * hc.lin_heads]
    W, U = hc.conv_width, len(L.segs)
    srcrows = torch.cat([qkv, cx_ext.to(qkv.dtype)]) if cx_ext is not None else qkv
    ok = (L.ctx_idx >= 0).unsqueeze(-1)
    ctx = srcrows.index_select(0, L.ctx_idx.clamp_min(0).reshape(-1)).view(U, W - 1, -1)
    cdt = torch.float64 if x.dtype == torch.float64 else torch.float32  # as linear_layer_forward
    ctx = torch.where(ok, ctx.to(cdt), torch.zeros((), device=x.device, dtype=cdt))
    qc = causal_conv(qkv, hw.fp32[f"layers.{i}.conv_w"].to(cdt), None, L.segs, ctx=ctx, ctx_idx=list(range(U)))
    C, Hh, d = hc.lin_width, hc.lin_heads, hc.lin_dim
    T = x.shape[0]
    q = torch.nn.functional.normalize(qc[:, :C].float().view(T, Hh, d), dim=-1).to(x.dtype).reshape(T, C)
    k = torch.nn.functional.normalize(qc[:, C:2 * C].float().view(T, Hh, d), dim=-1).to(x.dtype).reshape(T, C)
    v = qc[:, 2 * C:].contiguous()
    gd = torch.float64 if x.dtype == torch.float64 else torch.float32
    beta = torch.sigmoid(bb.to(gd))
    g = -torch.exp(hw.fp32[f"layers.{i}.A_log"].to(gd)) * torch.nn.functional.softplus(
        aa.to(gd) + hw.fp32[f"layers.{i}.dt_bias"].to(gd))
    q, k, g, beta = q.contiguous(), k.contiguous(), g.contiguous(), beta.contiguous()
    o = torch.zeros_like(v)
    fins = []
    for rows, segs, init in L.levels:
        pool = [st_ext] if st_ext is not None else []
        pool += fins
        init_state = torch.cat(pool) if pool and any(j >= 0 for j in init) else None
        oo, fin = recurrence(q.index_select(0, rows), k.index_select(0, rows), v.index_select(0, rows),
                             g.index_select(0, rows), beta.index_select(0, rows), segs, d ** -0.5, hc.kind == "gdn",
                             init_state=init_state, init_idx=init if init_state is not None else None)
        o = o.index_copy(0, rows, oo)
        fins.append(fin)
    st_keep = torch.cat(fins).index_select(0, L.own_fin) if len(L.own_fin) else None
    o = _rmsnorm_heads(o.view(T, Hh, d), t[f"layers.{i}.lin_norm"], cfg.rms_eps).reshape(T, C)
    o = (o.float() * torch.nn.functional.silu(z.float())).to(x.dtype)
    x = ops.linear(o, t[f"layers.{i}.lin_out"], None, residual=x)
    h2 = ops.rmsnorm(x, t[f"layers.{i}.ln2"], cfg.rms_eps, cfg.norm_plus_one)
    act = ops.swiglu(ops.linear(h2, t[f"layers.{i}.gu_w"]))
    y = ops.linear(act, t[f"layers.{i}.down_w"], None, residual=x)
    cx_keep = qkv.index_select(0, L.own_conv) if len(L.own_conv) else None
    return y, st_keep, cx_keep


def _chunk_layer(x, k_ext, v_ext, w, cfg, pos, plan, own, lw):
    """One decoder layer of a chunk whose keys continue with kept rows (k_ext, v_ext);
    returns (layer output, the k / v rows it keeps for later chunks)."""
    ln1, qkv_w, qkv_b, o_w, ln2, gu_w, down_w = w
    la = lw if lw is not None else (None, None, None, None)
    Hq, Hkv, D = cfg.heads, cfg.kv_heads, cfg.head_dim
    h = ops.rmsnorm(x, ln1, cfg.rms_eps, cfg.norm_plus_one)
    qkv = qkv_rope(h, qkv_w, qkv_b, pos, cfg, la[0])
    q, k, v = qkv[:, : Hq * D], qkv[:, Hq * D: (Hq + Hkv) * D], qkv[:, (Hq + Hkv) * D:]
    if k_ext is not None:
        ka, va = torch.cat([k, k_ext]), torch.cat([v, v_ext])
    else:
        ka, va = k.contiguous(), v.contiguous()
    a = ops.attention_kv(q, ka, va, plan, Hq, Hkv, D)
    x = ops.linear(a, o_w, None, residual=x, lora=la[1])
    h2 = ops.rmsnorm(x, ln2, cfg.rms_eps, cfg.norm_plus_one)
    act = ops.swiglu(ops.linear(h2, gu_w, lora=la[2]))
    y = ops.linear(act, down_w, None, residual=x, lora=la[3])
    return y, k.index_select(0, own), v.index_select(0, own)


class _LayerCkpt(torch.autograd.Function):
    """Checkpoint of a chunk layer fn(x, a_ext, b_ext, *args) -> (y, a_keep, b_keep) with
    three differentiable inputs and three outputs (attention: kept k / v rows; linear
    recurrence: kept states / conv input rows)."""

    @staticmethod
    def forward(ctx, x, k_ext, v_ext, fn, *args):
        ctx.fn, ctx.args = fn, args
        ctx.save_for_backward(x, k_ext, v_ext)
        with torch.no_grad():
            return fn(x, k_ext, v_ext, *args)

    @staticmethod
    def backward(ctx, dy, dk, dv):
        x, ke, ve = ctx.saved_tensors
        xr = x.detach().requires_grad_(True)
        ker = ke.detach().requires_grad_(True) if ke is not None else None
        ver = ve.detach().requires_grad_(True) if ve is not None else None
        with torch.enable_grad():
            y, kk, vk = ctx.fn(xr, ker, ver, *ctx.args)
        outs, grads = [y], [dy]
        for t, g in ((kk, dk), (vk, dv)):
            if t is not None and g is not None and t.numel():
                outs.append(t)
                grads.append(g)
        torch.autograd.backward(outs, grads)
        return (xr.grad, None if ker is None else ker.grad, None if ver is None else ver.grad) + \
            (None,) * (1 + len(ctx.args))


def _layer_slots(model, d: _DevChunk, i: int):
    """(ext index a, ext index b, own slots a, own slots b) of layer i in chunk d: attention
    layers read / keep k and v rows (one index for both); linear layers states and conv
    input rows."""
    if d.lin is not None and model.hc.is_linear(i):
        L = d.lin
        return L.ext_state, L.ext_conv, L.st, L.cx
    return d.ext, d.ext, (d.lo, d.hi), (d.lo, d.hi)


def _run_chunk(model, d: _DevChunk, kept_a, kept_b, temperature, lora, grad: bool):
    """A chunk through the model: ((logp, entropy) of its pairs, [(layer, a_keep, b_keep)],
    [(layer, a_ext, b_ext)] (leaves with gradients when grad))."""
    hybrid = hasattr(model, "hc")
    dense = model.dense if hybrid else model
    cfg = dense.cfg
    x = ops.embed(d.ids, dense["embed"])
    if grad and not x.requires_grad:
        x.requires_grad_(True)
    keeps, exts = [], []
    for i in range(cfg.layers):
        ia, ib, _, _ = _layer_slots(model, d, i)
        ae = kept_a[i].index_select(0, ia) if ia.numel() else None
        be = kept_b[i].index_select(0, ib) if ib.numel() else None
        for t in (ae, be):
            if grad and t is not None:
                t.requires_grad_(True)
        if hybrid and model.hc.is_linear(i):
            args = (_chunk_linear_layer, model, i, d.lin)
        else:
            args = (_chunk_layer, dense.layer(i), cfg, d.pos, d.plan, d.own,
                    lora.layer(i) if lora is not None else None)
        if grad:
            x, ka, kb = _LayerCkpt.apply(x, ae, be, *args)
        else:
            x, ka, kb = args[0](x, ae, be, *args[1:])
        keeps.append((i, ka, kb))
        exts.append((i, ae, be))
    h = ops.rmsnorm(x, dense["norm"], cfg.rms_eps, cfg.norm_plus_one)
    hp = h.index_select(0, d.pair_local)
    out = ops.logprob_head(hp, dense.head, d.labels, 1.0 / temperature, cfg.vocab_size)
    return out, keeps, exts


def _kept_sizes(model, plan, i: int) -> tuple[int, int]:
    if getattr(plan, "linear", None) is not None and model.hc.is_linear(i):
        return plan.linear.n_state, plan.linear.n_conv
    return plan.n_kept, plan.n_kept


class _ChunkMajor(torch.autograd.Function):
    @staticmethod
    def forward(ctx, anchor, model, plan, temperature, lora, device):
        dense = model.dense if hasattr(model, "hc") else model
        cfg = dense.cfg
        dt = dense["embed"].dtype
        kept_a, kept_b = [None] * cfg.layers, [None] * cfg.layers
        fdt = torch.float64 if dt == torch.float64 else torch.float32
        logp = torch.zeros(plan.n_pairs, dtype=fdt, device=device)
        ent = torch.zeros_like(logp)
        devs = [_DevChunk(plan, ch, device, c) for c, ch in enumerate(plan.chunks)]
        with torch.no_grad():
            for d in devs:
                (lp, en), keeps, _ = _run_chunk(model, d, kept_a, kept_b, temperature, lora, grad=False)
                logp[d.pair_idx] = lp.to(fdt)
                ent[d.pair_idx] = en.to(fdt)
                for i, ka, kb in keeps:
                    _, _, (alo, ahi), (blo, bhi) = _layer_slots(model, d, i)
                    na, nb = _kept_sizes(model, plan, i)
                    if ahi > alo:
                        if kept_a[i] is None:  # allocated at the first write: shape / dtype of what is kept
                            kept_a[i] = torch.empty((na,) + tuple(ka.shape[1:]), dtype=ka.dtype, device=device)
                        kept_a[i][alo:ahi] = ka
                    if bhi > blo:
                        if kept_b[i] is None:
                            kept_b[i] = torch.empty((nb,) + tuple(kb.shape[1:]), dtype=kb.dtype, device=device)
                        kept_b[i][blo:bhi] = kb
        ctx.state = (model, plan, temperature, lora, devs, kept_a, kept_b)
        return logp, ent

    @staticmethod
    def backward(ctx, g_logp, g_ent):
        model, plan, temperature, lora, devs, kept_a, kept_b = ctx.state

        def zeros(t):
            if t is None:
                return None
            return torch.zeros(t.shape, dtype=torch.promote_types(t.dtype, torch.float32), device=t.device)
        sums_a, sums_b = [zeros(t) for t in kept_a], [zeros(t) for t in kept_b]
        g_logp = g_logp if g_logp is not None else torch.zeros(plan.n_pairs, device=devs[0].ids.device)
        g_ent = g_ent if g_ent is not None else torch.zeros_like(g_logp)
        for d in reversed(devs):
            with torch.enable_grad():
                (lp, en), keeps, exts = _run_chunk(model, d, kept_a, kept_b, temperature, lora, grad=True)
                outs = [lp, en]
                grads = [g_logp.index_select(0, d.pair_idx).to(lp.dtype),
                         g_ent.index_select(0, d.pair_idx).to(en.dtype)]
                for i, ka, kb in keeps:
                    _, _, (alo, ahi), (blo, bhi) = _layer_slots(model, d, i)
                    if ahi > alo and ka is not None:
                        outs.append(ka)
                        grads.append(sums_a[i][alo:ahi].to(ka.dtype))
                    if bhi > blo and kb is not None:
                        outs.append(kb)
                        grads.append(sums_b[i][blo:bhi].to(kb.dtype))
                torch.autograd.backward(outs, grads)
            for i, ae, be in exts:
                ia, ib, _, _ = _layer_slots(model, d, i)
                if ae is not None and ae.grad is not None:
                    sums_a[i].index_add_(0, ia, ae.grad.to(sums_a[i].dtype))
                if be is not None and be.grad is not None:
                    sums_b[i].index_add_(0, ib, be.grad.to(sums_b[i].dtype))
        ctx.state = None
        return None, None, None, None, None, None


def chunk_major_forward(weights, mb, tokens: int, temperature: float = 1.0, lora=None, device=None):
    """(logp [pairs], entropy [pairs]) of micro-batch `mb` (rl.actor.MicroBatch) computed
    chunk-major with chunks of at most `tokens` tree rows; differentiable (the backward runs
    the chunks in reverse and accumulates parameter gradients into main_grad).  `weights`:
    decoder Weights, or models.hybrid.HybridWeights (linear layers keep states and conv
    rows across chunks)."""
    dense = weights.dense if hasattr(weights, "hc") else weights
    device = device or dense["embed"].device
    plan = ChunkPlan(mb, tokens)
    if hasattr(weights, "hc"):
        plan.linear = _LinearPlan(plan, mb, weights.hc.conv_width)
    anchor = torch.zeros((), device=device, requires_grad=torch.is_grad_enabled())
    return _ChunkMajor.apply(anchor, weights, plan, temperature, lora, device)


__all__ = ["ChunkPlan", "chunk_major_forward"]
