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
the kept rows it reads].

run_forward runs the chunks in order without autograd (keeping what later chunks read);
run_backward runs them in reverse with autograd: each layer is checkpointed, its inputs
being the layer input and the kept k / v it reads, so the recompute returns their
gradients, which are summed (fp32) into the owning chunk's slots; when that chunk runs,
the sums are the output gradients of the k / v it kept.  Parameter gradients add up to
those of the whole tree (they accumulate in the weights' main_grad buffers).
chunk_major_forward is both as one autograd op returning (logp, entropy) per scored pair.

Reference parity (behaviour): `octopus/rl/chunk_major.py:1-40` (chunk order, kept tensors,
reverse-chunk backward with gradient sums, one autograd op), `ChunkPlan` (`:73-168`),
`run_forward` / `run_backward` (`:326-363`); the dense decoder only here (the reference
also keeps recurrent states and convolution context rows for hybrid models).
"""
from __future__ import annotations

import heapq
from dataclasses import dataclass

import numpy as np
import torch

from .. import ops


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

    def __init__(self, plan: ChunkPlan, ch: Chunk, device):
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


def _chunk_layer(x, k_ext, v_ext, w, cfg, pos, plan, own, lw):
    """One decoder layer of a chunk whose keys continue with kept rows (k_ext, v_ext);
    returns (layer output, the k / v rows it keeps for later chunks)."""
    ln1, qkv_w, qkv_b, o_w, ln2, gu_w, down_w = w
    la = lw if lw is not None else (None, None, None, None)
    Hq, Hkv, D = cfg.heads, cfg.kv_heads, cfg.head_dim
    h = ops.rmsnorm(x, ln1, cfg.rms_eps, cfg.norm_plus_one)
    qkv = ops.linear(h, qkv_w, qkv_b, lora=la[0])
    qkv = ops.rope_(qkv, pos, Hq, Hkv, D, cfg.rope_theta)
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
    """Checkpoint of _chunk_layer with three differentiable inputs (x, k_ext, v_ext) and
    three outputs (y, kept k, kept v)."""

    @staticmethod
    def forward(ctx, x, k_ext, v_ext, *args):
        ctx.args = args
        ctx.save_for_backward(x, k_ext, v_ext)
        with torch.no_grad():
            return _chunk_layer(x, k_ext, v_ext, *args)

    @staticmethod
    def backward(ctx, dy, dk, dv):
        x, ke, ve = ctx.saved_tensors
        xr = x.detach().requires_grad_(True)
        ker = ke.detach().requires_grad_(True) if ke is not None else None
        ver = ve.detach().requires_grad_(True) if ve is not None else None
        with torch.enable_grad():
            y, kk, vk = _chunk_layer(xr, ker, ver, *ctx.args)
        outs, grads = [y], [dy]
        for t, g in ((kk, dk), (vk, dv)):
            if g is not None and t.numel():
                outs.append(t)
                grads.append(g)
        torch.autograd.backward(outs, grads)
        return (xr.grad, None if ker is None else ker.grad, None if ver is None else ver.grad) + (None,) * len(ctx.args)


def _run_chunk(weights, d: _DevChunk, kept_k, kept_v, temperature, lora, grad: bool):
    """A chunk through the model: ((logp, entropy) of its pairs, [(layer, k_keep, v_keep)],
    [(layer, k_ext, v_ext)] (leaves with gradients when grad))."""
    cfg = weights.cfg
    x = ops.embed(d.ids, weights["embed"])
    if grad and not x.requires_grad:
        x.requires_grad_(True)
    keeps, exts = [], []
    for i in range(cfg.layers):
        ke = ve = None
        if d.ext.numel():
            ke = kept_k[i].index_select(0, d.ext)
            ve = kept_v[i].index_select(0, d.ext)
            if grad:
                ke.requires_grad_(True)
                ve.requires_grad_(True)
        args = (weights.layer(i), cfg, d.pos, d.plan, d.own, lora.layer(i) if lora is not None else None)
        if grad:
            x, kk, vk = _LayerCkpt.apply(x, ke, ve, *args)
        else:
            x, kk, vk = _chunk_layer(x, ke, ve, *args)
        keeps.append((i, kk, vk))
        exts.append((i, ke, ve))
    h = ops.rmsnorm(x, weights["norm"], cfg.rms_eps, cfg.norm_plus_one)
    hp = h.index_select(0, d.pair_local)
    out = ops.logprob_head(hp, weights.head, d.labels, 1.0 / temperature, cfg.vocab_size)
    return out, keeps, exts


class _ChunkMajor(torch.autograd.Function):
    @staticmethod
    def forward(ctx, anchor, weights, plan, temperature, lora, device):
        cfg = weights.cfg
        W = cfg.kv_heads * cfg.head_dim
        dt = weights["embed"].dtype
        kept_k = [torch.empty(plan.n_kept, W, dtype=dt, device=device) for _ in range(cfg.layers)]
        kept_v = [torch.empty(plan.n_kept, W, dtype=dt, device=device) for _ in range(cfg.layers)]
        fdt = torch.float64 if dt == torch.float64 else torch.float32
        logp = torch.zeros(plan.n_pairs, dtype=fdt, device=device)
        ent = torch.zeros_like(logp)
        devs = [_DevChunk(plan, ch, device) for ch in plan.chunks]
        with torch.no_grad():
            for d in devs:
                (lp, en), keeps, _ = _run_chunk(weights, d, kept_k, kept_v, temperature, lora, grad=False)
                logp[d.pair_idx] = lp.to(fdt)
                ent[d.pair_idx] = en.to(fdt)
                for i, kk, vk in keeps:
                    if d.hi > d.lo:
                        kept_k[i][d.lo:d.hi] = kk
                        kept_v[i][d.lo:d.hi] = vk
        ctx.state = (weights, plan, temperature, lora, devs, kept_k, kept_v)
        return logp, ent

    @staticmethod
    def backward(ctx, g_logp, g_ent):
        weights, plan, temperature, lora, devs, kept_k, kept_v = ctx.state
        cfg = weights.cfg
        acc = torch.promote_types(kept_k[0].dtype, torch.float32) if kept_k else torch.float32
        sums_k = [torch.zeros(t.shape, dtype=acc, device=t.device) for t in kept_k]
        sums_v = [torch.zeros(t.shape, dtype=acc, device=t.device) for t in kept_v]
        g_logp = g_logp if g_logp is not None else torch.zeros(plan.n_pairs, device=devs[0].ids.device)
        g_ent = g_ent if g_ent is not None else torch.zeros_like(g_logp)
        for d in reversed(devs):
            with torch.enable_grad():
                (lp, en), keeps, exts = _run_chunk(weights, d, kept_k, kept_v, temperature, lora, grad=True)
                outs = [lp, en]
                grads = [g_logp.index_select(0, d.pair_idx).to(lp.dtype), g_ent.index_select(0, d.pair_idx).to(en.dtype)]
                if d.hi > d.lo:
                    for i, kk, vk in keeps:
                        outs += [kk, vk]
                        grads += [sums_k[i][d.lo:d.hi].to(kk.dtype), sums_v[i][d.lo:d.hi].to(vk.dtype)]
                torch.autograd.backward(outs, grads)
            for i, ke, ve in exts:
                if ke is not None:
                    sums_k[i].index_add_(0, d.ext, ke.grad.to(acc))
                    sums_v[i].index_add_(0, d.ext, ve.grad.to(acc))
        ctx.state = None
        return None, None, None, None, None, None


def chunk_major_forward(weights, mb, tokens: int, temperature: float = 1.0, lora=None, device=None):
    """(logp [pairs], entropy [pairs]) of micro-batch `mb` (rl.actor.MicroBatch) computed
    chunk-major with chunks of at most `tokens` tree rows; differentiable (the backward runs
    the chunks in reverse and accumulates parameter gradients into main_grad)."""
    device = device or weights["embed"].device
    plan = ChunkPlan(mb, tokens)
    anchor = torch.zeros((), device=device, requires_grad=torch.is_grad_enabled())
    return _ChunkMajor.apply(anchor, weights, plan, temperature, lora, device)


__all__ = ["ChunkPlan", "chunk_major_forward"]
