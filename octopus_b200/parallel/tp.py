"""Tensor parallelism of the rollout engine (Megatron-style column/row split with
sequence-parallel activations), on fused compute + collective kernels over NVLink.

Layout per TP rank r of tp (heads and FFN columns split evenly):

  qkv_w   rows [q heads of r | k heads of r | v heads of r]     column-parallel (AG -> GEMM)
  o_w     columns of r's q heads                              row-parallel    (GEMM -> RS)
  gu_w    rows [gate F/tp of r | up F/tp of r]                 column-parallel (AG -> GEMM)
  down_w  columns F/tp of r                                   row-parallel    (GEMM -> RS)
  head    vocabulary rows [r V/tp, (r+1) V/tp)                vocab-parallel sampling
  embed, norms                                                replicated (views of the trainer's)

Between the row- and column-parallel GEMMs the residual stream is sequence-sharded:
rank r keeps rows [r rows_s, (r+1) rows_s) of h.  One layer on rank r:

  x_r  = rmsnorm(h_r)                      (written into r's IPC activation buffer)
  qkv  = AG(x_0..x_tp-1) @ qkv_w_r^T       ag_gemm: peer rows copied into local staging, tcgen05 MMA
  o    = attention(rope(qkv)) on r's heads  local KV cache holds r's KV heads
  h_r += RS(o @ o_w_r^T)                   gemm_rs: epilogue peer stores + tp_reduce
  x_r  = rmsnorm(h_r)                      (fused into tp_reduce)
  gu   = AG(x) @ gu_w_r^T;  a = swiglu(gu)
  h_r += RS(a @ down_w_r^T); x_r = rmsnorm_next(h_r)

and sampling is a vocab-parallel Gumbel-max over r's vocabulary rows followed by an
exchange of 4 floats per row, so every rank ends with the same tokens.

Synchronisation (all inside the kernels, no host sequence numbers, CUDA-graph safe):
counters in a small IPC sync buffer per rank (see csrc/tp.h); every forward starts with
a bounded barrier so no rank overwrites a buffer a peer may still read from the
previous forward.  Within a forward, the alternation of AG and RS orders every buffer
reuse: a rank rewrites its activation shard only after the reduce that waited for
every peer's RS signal, which each peer sent after its AG finished reading.

Reference parity: the reference's rollout TP is SGLang's (`--tp`), configured by
`octopus/rl/grpo.yaml` (`rollout` section); SGLang runs NCCL all-reduce after each
row-parallel layer.  The weight sync to the TP layout replaces SGLang's
update-weights path used by `octopus/rl/train.py:121-133`.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch
import torch.distributed as dist

from .. import ops

SLOT_AG, SLOT_RS, SLOT_SMP, SLOT_BAR = 0, 1, 2, 3


def tp_rows(n: int) -> int:
    """Rows per rank the fused kernels accept: 8, 16, 32, 64 or a multiple of 128."""
    for r in (8, 16, 32, 64, 128):
        if n <= r:
            return r
    return (n + 127) // 128 * 128


# ------------------------------------------------------------------------ shard layout
@dataclass
class ShardDims:
    tp: int
    rank: int
    hq: int          # local query heads
    hkv: int         # local KV heads
    d: int
    f: int           # local FFN width
    v: int           # local vocabulary rows
    col_base: int    # first global vocabulary index of this rank
    vocab_limit: int  # valid local vocabulary rows

    @property
    def q_loc(self):
        return self.hq * self.d

    @property
    def kv_loc(self):
        return self.hkv * self.d

    @property
    def qkv_loc(self):
        return self.q_loc + 2 * self.kv_loc


def shard_dims(cfg, tp: int, rank: int) -> ShardDims:
    if cfg.heads % tp or cfg.kv_heads % tp or cfg.ffn % tp:
        raise ValueError(f"tp={tp} must divide heads {cfg.heads}, kv heads {cfg.kv_heads} and ffn {cfg.ffn}")
    V = cfg.vocab_size
    vs = (V + tp - 1) // tp
    vs = (vs + 7) // 8 * 8
    base = rank * vs
    return ShardDims(tp, rank, cfg.heads // tp, cfg.kv_heads // tp, cfg.head_dim, cfg.ffn // tp, vs, base,
                     max(0, min(vs, V - base)))


def shard_segments(cfg, w, sd: ShardDims):
    """(name, [(src view, dst slice spec)]) of every sharded matrix: each entry is a
    2D source view of the trainer's tensor and the destination shape."""
    H, D = cfg.hidden, cfg.head_dim
    r = sd.rank
    out = []
    for i in range(cfg.layers):
        qkv = w[f"layers.{i}.qkv_w"]
        q0 = r * sd.q_loc
        k0 = cfg.q_width + r * sd.kv_loc
        v0 = cfg.q_width + cfg.kv_width + r * sd.kv_loc
        out.append((f"layers.{i}.qkv_w", [qkv[q0:q0 + sd.q_loc], qkv[k0:k0 + sd.kv_loc], qkv[v0:v0 + sd.kv_loc]],
                    (sd.qkv_loc, H)))
        if cfg.qkv_bias:
            b = w[f"layers.{i}.qkv_b"][None, :]
            out.append((f"layers.{i}.qkv_b", [b[:, q0:q0 + sd.q_loc], b[:, k0:k0 + sd.kv_loc],
                                              b[:, v0:v0 + sd.kv_loc]], (1, sd.qkv_loc)))
        o = w[f"layers.{i}.o_w"]
        out.append((f"layers.{i}.o_w", [o[:, r * sd.q_loc:(r + 1) * sd.q_loc]], (H, sd.q_loc)))
        gu = w[f"layers.{i}.gu_w"]
        F = cfg.ffn
        out.append((f"layers.{i}.gu_w", [gu[r * sd.f:(r + 1) * sd.f], gu[F + r * sd.f:F + (r + 1) * sd.f]],
                    (2 * sd.f, H)))
        dn = w[f"layers.{i}.down_w"]
        out.append((f"layers.{i}.down_w", [dn[:, r * sd.f:(r + 1) * sd.f]], (H, sd.f)))
    return out


class TPWeights:
    """This rank's TP shards in one contiguous buffer, refreshed from the trainer's
    weights by the reshard kernel (one launch for all matrices)."""

    def __init__(self, cfg, full, sd: ShardDims, device):
        self.cfg, self.full, self.sd = cfg, full, sd
        self.device = torch.device(device)
        segs = shard_segments(cfg, full, sd)
        total = 0
        self.offsets = {}
        for name, _, shape in segs:
            self.offsets[name] = total
            total += math.prod(shape)
            total = (total + 255) // 256 * 256
        self.flat = torch.empty(total, dtype=full.flat.dtype, device=self.device)
        self.t = {}
        self._copies = []  # (source view, destination view): row blocks, or column blocks of a bias
        for name, srcs, shape in segs:
            o = self.offsets[name]
            dst = self.flat[o:o + math.prod(shape)].view(shape)
            self.t[name] = dst if name.endswith("_w") else dst[0]
            a = 0
            for s in srcs:
                if shape[0] == 1:
                    self._copies.append((s, dst[:, a:a + s.shape[1]]))
                    a += s.shape[1]
                else:
                    self._copies.append((s, dst[a:a + s.shape[0]]))
                    a += s.shape[0]
        self._segs = None
        if self.device.type == "cuda":
            self._segs, self._chunks = self._build_segments()
        self.refresh()

    def _build_segments(self):
        rows, first = [], 0
        for s, d in self._copies:
            n_rows, n_cols = s.shape
            if (n_cols % 8 or s.stride(1) != 1 or d.stride(1) != 1 or s.data_ptr() % 16 or d.data_ptr() % 16
                    or (n_rows > 1 and (s.stride(0) % 8 or d.stride(0) % 8))):
                raise ValueError("reshard: 16-byte aligned rows of a multiple of 8 elements required")
            rows.append([s.data_ptr(), d.data_ptr(), s.stride(0), d.stride(0), n_rows | (n_cols << 32), first])
            first += n_rows * (n_cols // 8)
        t = torch.tensor(np.asarray(rows, dtype=np.int64), device=self.device)
        return t, first

    def refresh(self):
        """Weight sync: trainer layout -> TP shards."""
        if self._segs is not None:
            ops.ext().reshard_copy(self._segs, self._chunks)
            ops.add_launches(1)
        else:
            for s, d in self._copies:
                d.copy_(s)

    def layer(self, i):
        cfg = self.cfg
        b = self.t.get(f"layers.{i}.qkv_b")
        return (self.full[f"layers.{i}.ln1"], self.t[f"layers.{i}.qkv_w"], b, self.t[f"layers.{i}.o_w"],
                self.full[f"layers.{i}.ln2"], self.t[f"layers.{i}.gu_w"], self.t[f"layers.{i}.down_w"])

    @property
    def head(self):
        h = self.full.head
        sd = self.sd
        return h[sd.col_base: sd.col_base + sd.vocab_limit]


# ------------------------------------------------------------------------ communicator
class TPGroup:
    """IPC buffers and fused kernels of one TP group (one process per GPU)."""

    def __init__(self, group, device, *, max_rows: int, hidden: int, max_n: int, max_sample_rows: int):
        from .peer import PeerBuffers

        self.group = group
        self.tp = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = torch.device(device)
        self.hidden = hidden
        self.max_rows_s = tp_rows((max_rows + self.tp - 1) // self.tp)
        C = ops.ext()
        self.sync = PeerBuffers(C.tp_sync_bytes(), self.device, group)
        self.xbuf = PeerBuffers(self.max_rows_s * hidden * 2, self.device, group)
        # RS receive slots: [splits * tp][rows][N]; decode-sized calls may use up to 8 K splits
        self.recv_elems = self.tp * max(self.max_rows_s, 8 * 256 // self.tp) * max_n
        self.recv = PeerBuffers(self.recv_elems * 2, self.device, group)
        self.max_sel = tp_rows(max_sample_rows)
        self.sel = PeerBuffers(self.max_sel * hidden * 2, self.device, group)
        max_m = self.tp * max(self.max_sel, self.max_rows_s)  # rows of one sampling call
        self.xch = PeerBuffers(self.tp * max_m * 16, self.device, group)
        self.max_n = max_n
        self.sync_local = self.sync.ptrs[self.rank]
        # AG staging: every remote activation row is copied over NVLink once per GEMM
        max_m = self.tp * max(self.max_rows_s, self.max_sel)
        self.stage = torch.empty(max_m * hidden, dtype=torch.bfloat16, device=self.device)
        self.work = torch.zeros(2 + max_m // 128 + 1, dtype=torch.int32, device=self.device)

    # ------------------------------------------------------------------ views
    def x_local(self, rows_s: int) -> torch.Tensor:
        return self.xbuf.local.view(torch.bfloat16)[: rows_s * self.hidden].view(rows_s, self.hidden)

    def sel_local(self, rows_s: int) -> torch.Tensor:
        return self.sel.local.view(torch.bfloat16)[: rows_s * self.hidden].view(rows_s, self.hidden)

    def recv_local(self, rows_s: int, n: int, splits: int = 1) -> torch.Tensor:
        return self.recv.local.view(torch.bfloat16)[: splits * self.tp * rows_s * n]

    # ------------------------------------------------------------------ kernels
    def barrier(self):
        ops.ext().tp_barrier(self.rank, self.sync_local, self.sync.ptrs, SLOT_BAR, self.device.index)
        ops.add_launches(1)

    def ag_linear(self, rows_s: int, W, out, bias=None, sel: bool = False):
        bufs = self.sel if sel else self.xbuf
        ops.ext().ag_gemm(bufs.ptrs, rows_s, self.hidden, W, out, bias, self.rank, self.sync_local, self.sync.ptrs,
                          SLOT_AG, 0, self.stage, self.work)
        ops.add_launches(2 if self.tp * rows_s <= 256 else 1)  # (+ split-K finish for decode sizes)
        return out

    def rs_linear(self, a, W):
        """Returns the call's (grid, splits): what the owners' reduce consumes."""
        n = W.shape[0]
        if n > self.max_n or a.shape[0] > self.tp * self.max_rows_s:
            raise ValueError("gemm_rs: output larger than the receive buffers")
        ops.add_launches(1)
        g, sp = ops.ext().gemm_rs(a, W, self.recv.ptrs, self.recv_elems, self.rank, self.sync_local, self.sync.ptrs,
                                  SLOT_RS, 0)
        return g, sp

    def reduce(self, h, call, w=None, x=None, eps: float = 1e-6, plus_one: bool = False):
        grid, splits = call
        rows_s, n = h.shape
        ops.ext().tp_reduce(self.recv_local(rows_s, n, splits), splits, h, w, x, eps, plus_one, self.rank,
                            self.sync_local, self.sync.ptrs, SLOT_RS, grid)
        ops.add_launches(1)

    def sample(self, rows_s: int, W, temperature: float, seed: int, streams, sd: ShardDims, sel: bool = False):
        bufs = self.sel if sel else self.xbuf
        alpha = 1.0 / max(temperature, 1e-6)
        ops.add_launches(3)
        return ops.ext().tp_sample_head(bufs.ptrs, rows_s, self.hidden, W, alpha, seed, streams, sd.vocab_limit,
                                        sd.col_base, self.rank, self.sync_local, self.sync.ptrs, SLOT_AG, SLOT_SMP,
                                        self.xch.ptrs, self.xch.local, self.stage, self.work)

    def close(self):
        torch.cuda.synchronize(self.device)
        for b in (self.sync, self.xbuf, self.recv, self.sel, self.xch):
            b.close()


# ------------------------------------------------------------------------ CPU reference
def reference_layer(cfg, full, tp: int, x, pos, attn_fn):
    """fp32 emulation of one TP layer over `tp` virtual ranks (shard slicing + rank-order
    reduction), for checking the shard layout on CPU.  attn_fn(q, k, v, hq, hkv) -> o."""
    from ..ops import reference as ref

    H = cfg.hidden
    f = lambda t: t.float()
    dims = [shard_dims(cfg, tp, r) for r in range(tp)]
    segs = [dict((n, (s, shp)) for n, s, shp in shard_segments(cfg, full, d)) for d in dims]
    h = f(x)
    i = 0
    xn = ref.rmsnorm(h, full[f"layers.{i}.ln1"], cfg.rms_eps, cfg.norm_plus_one).float()
    parts = []
    for r, sd in enumerate(dims):
        wq = torch.cat([f(s) for s in segs[r][f"layers.{i}.qkv_w"][0]])
        qkv = xn @ wq.t()
        if cfg.qkv_bias:
            qkv = qkv + torch.cat([f(s) for s in segs[r][f"layers.{i}.qkv_b"][0]], dim=1)[0]
        q, k, v = qkv[:, :sd.q_loc], qkv[:, sd.q_loc:sd.q_loc + sd.kv_loc], qkv[:, sd.q_loc + sd.kv_loc:]
        o = attn_fn(q, k, v, sd.hq, sd.hkv, pos)
        parts.append(o @ f(segs[r][f"layers.{i}.o_w"][0][0]).t())
    h = h + sum(parts)
    xn = ref.rmsnorm(h, full[f"layers.{i}.ln2"], cfg.rms_eps, cfg.norm_plus_one).float()
    parts = []
    for r, sd in enumerate(dims):
        wgu = torch.cat([f(s) for s in segs[r][f"layers.{i}.gu_w"][0]])
        a = ref.swiglu(xn @ wgu.t())
        parts.append(a @ f(segs[r][f"layers.{i}.down_w"][0][0]).t())
    return h + sum(parts)
