"""Paged decode attention (one query row per request) over page-size-1 KV slots.

The KV cache of a layer is ``k_cache, v_cache: [slots, Hkv, D]``; request b reads the
slots ``kv_indices[kv_indptr[b]:kv_indptr[b+1]]`` (its own pages, shared-prefix pages
and mounted pages alike).  The CUDA path is a split-K kernel; its partial results go
to a scratch buffer owned by :class:`DecodeAttention` so the call is CUDA-graph safe.
Reference parity: SGLang's Triton decode backend as used by
`octopus/serving/kv_mount.py:585-634` (per-layer KV views over kv_indptr/kv_indices).
"""
from __future__ import annotations

import math

import torch

from . import reference as ref
from ._ext import ext


class DecodeAttention:
    """Holds the split-K scratch for batches up to ``max_batch`` requests."""

    def __init__(self, Hq: int, Hkv: int, D: int, max_batch: int, num_splits: int = 8, device="cuda",
                 persistent: bool | None = None):
        self.Hq, self.Hkv, self.D = Hq, Hkv, D
        # the persistent producer/consumer kernel covers head_dim 128 (all BASELINE models)
        self.persistent = (D == 128) if persistent is None else persistent
        self.num_splits = num_splits
        self.max_batch = max_batch
        dev = torch.device(device)
        if dev.type == "cuda" and num_splits > 1:
            self.part_o = torch.empty(max_batch * Hq * num_splits * D, dtype=torch.float32, device=dev)
            self.part_lse = torch.empty(max_batch * Hq * num_splits, dtype=torch.float32, device=dev)
        else:
            self.part_o = torch.empty(0, dtype=torch.float32, device=dev)
            self.part_lse = torch.empty(0, dtype=torch.float32, device=dev)

    def __call__(self, q, k_cache, v_cache, kv_indptr, kv_indices, out=None, scale=None, kv_len=None):
        """q: [B, Hq*D] -> o [B, Hq*D].

        Request b reads kv_indices[start[b] : start[b] + len[b]] where (start, len) are
        (kv_indptr[:-1], diff(kv_indptr)) or, when ``kv_len`` is given, (kv_indptr, kv_len).
        """
        B = q.shape[0]
        scale = scale if scale is not None else self.D ** -0.5
        if out is None:
            out = torch.empty(B, self.Hq * self.D, dtype=q.dtype, device=q.device)
        if kv_len is None:
            start, length = kv_indptr[:-1], kv_indptr[1:] - kv_indptr[:-1]
        else:
            start, length = kv_indptr, kv_len
        if q.is_cuda:
            assert B <= self.max_batch, "decode batch exceeds the scratch capacity"
            st, ln = start.to(torch.int32).contiguous(), length.to(torch.int32).contiguous()
            if self.persistent:
                ext().attn_decode_persistent(q, k_cache, v_cache, st, ln, kv_indices, out, self.part_o,
                                             self.part_lse, self.Hq, self.Hkv, self.num_splits, scale)
            else:
                ext().attn_decode(q, k_cache, v_cache, st, ln, kv_indices, out, self.part_o, self.part_lse,
                                  self.Hq, self.Hkv, self.D, self.num_splits, scale)
            return out
        return decode_attention_ref(q, k_cache, v_cache, start.cpu(), kv_indices, self.Hq, self.Hkv, self.D, scale,
                                    out, length.cpu())


def decode_attention_ref(q, k_cache, v_cache, kv_start, kv_indices, Hq, Hkv, D, scale, out=None, kv_len=None):
    """Reference; (kv_start, kv_len) or an indptr in kv_start when kv_len is None."""
    B = q.shape[0]
    if kv_len is None:
        st = kv_start[:-1].tolist()
        ln = (kv_start[1:] - kv_start[:-1]).tolist()
    else:
        st, ln = kv_start.tolist(), kv_len.tolist()
    res = torch.empty(B, Hq, D, dtype=torch.float32)
    for b in range(B):
        idx = kv_indices[st[b]:st[b] + ln[b]].long()
        o, _ = ref.gather_attention(q[b:b + 1].reshape(1, Hq, D), k_cache.reshape(-1, Hkv, D),
                                    v_cache.reshape(-1, Hkv, D), [0, 1], [0, len(idx)], idx, scale, causal=False)
        res[b] = o[0]
    r = res.reshape(B, Hq * D).to(q.dtype)
    if out is not None:
        out.copy_(r)
        return out
    return r


def decode_attention(q, k_cache, v_cache, kv_indptr, kv_indices, Hq, Hkv, D, scale=None, num_splits=8):
    return DecodeAttention(Hq, Hkv, D, q.shape[0], num_splits, q.device)(q, k_cache, v_cache, kv_indptr,
                                                                         kv_indices, scale=scale)


class SharedDecode:
    """Shared-prefix decode (cascade attention) with static device tables.

    `plan()` splits every row's key list into segments: key ranges identical across up
    to `seg_rows` rows (their contexts agree: a mounted task prefix, a forked parent's
    context) and each row's own remainder, whose length grows with decoding.  The
    kernel gathers a shared segment's K/V once for all its rows.  Tables are rewritten
    in place, so a CUDA graph captured once per batch bucket stays valid across plans.
    """

    SEG_STRIDE = 16  # rows per segment in the device tables (kSegRows)

    def __init__(self, Hq: int, Hkv: int, D: int, max_batch: int, device="cuda", max_slots: int = 32,
                 chunk: int | None = None, min_shared: int = 64, max_segs: int | None = None,
                 use_tc: bool | None = None):
        import os

        if D != 128:
            raise ValueError("shared-prefix decode covers head_dim 128")
        self.Hq, self.Hkv, self.D = Hq, Hkv, D
        G = Hq // Hkv
        # tcgen05 kernel: one MMA tile holds 128 / G rows' heads; mma.sync kernel: two warps of 16 / G.
        # The mma.sync kernel is the default: in the 7B DAG RL step it took 5.1 s of decode attention
        # against 6.4 s for the tcgen05 one (which wins only on consecutive-slot solver batches:
        # 121 vs 165 us); OCTO_DECODE_TC=1 selects the tcgen05 kernel.
        self.use_tc = (os.environ.get("OCTO_DECODE_TC", "0") != "0") if use_tc is None else bool(use_tc)
        self.seg_rows = min(self.SEG_STRIDE, 128 // G) if self.use_tc else min(8, 2 * (16 // G))
        # keys per work item: each item pays a descriptor / Q / partial-write overhead, which the
        # tcgen05 kernel amortises best over 1024 keys (7B DAG solver stage: 121 vs 145 us at 256)
        chunk = chunk or (1024 if self.use_tc else 256)
        self.max_batch, self.max_slots, self.chunk, self.min_shared = max_batch, max_slots, chunk, min_shared
        self.max_segs = max_segs or 6 * max_batch
        dev = torch.device(device)
        i32 = dict(dtype=torch.int32, device=dev)
        S = self.max_segs
        self.t_rows = torch.full((S * self.SEG_STRIDE,), -1, **i32)
        self.t_slot = torch.zeros(S * self.SEG_STRIDE, **i32)
        self.t_start = torch.zeros(S, **i32)
        self.t_len = torch.zeros(S, **i32)
        self.t_off = torch.zeros(S, **i32)
        self.t_items = torch.zeros(S * 64, **i32)
        self.t_n = torch.zeros(2, **i32)  # [work items, keys per item]
        sms = torch.cuda.get_device_properties(dev).multi_processor_count if dev.type == "cuda" else 148
        self.target_items = 4 * 2 * sms  # ~4 items per CTA of the persistent grid (2 CTAs per SM)
        self.t_nslot = torch.zeros(max_batch, **i32)
        self.part_o = torch.empty(max_batch * Hq * max_slots * D, dtype=torch.float32, device=dev)
        self.part_lse = torch.empty(max_batch * Hq * max_slots, dtype=torch.float32, device=dev)
        self.stats = {}

    def plan(self, lists: list, starts, ctx_len, final_len, B: int) -> bool:
        """lists[b]: row b's key slots (numpy, >= its final length); starts[b]: offset of that
        list in the kv index buffer; ctx_len[b]: leading keys that are context (may be
        shared); final_len[b]: the row's key count at the end of this decode call.  Rows
        past len(lists) are padding.  Returns False when the tables cannot hold the plan."""
        import numpy as np

        segs = []  # (rows, start, len (-1 dynamic), off, max_len)
        n = len(lists)

        def own(b, off):
            segs.append(([b], int(starts[b]) + off, -1, off, max(0, int(final_len[b]) - off)))

        def rec(rows, off):
            groups: dict = {}
            for b in rows:
                if ctx_len[b] <= off:
                    own(b, off)
                else:
                    groups.setdefault(int(lists[b][off]), []).append(b)
            for grp in groups.values():
                if len(grp) == 1:
                    own(grp[0], off)
                    continue
                m = min(int(ctx_len[b]) for b in grp)
                A = np.stack([np.asarray(lists[b][off:m]) for b in grp])
                neq = np.nonzero((A != A[0]).any(axis=0))[0]
                L = int(neq[0]) if len(neq) else m - off
                if L < self.min_shared:
                    for b in grp:
                        own(b, off)
                    continue
                for i in range(0, len(grp), self.seg_rows):
                    part = grp[i:i + self.seg_rows]
                    segs.append((part, int(starts[part[0]]) + off, L, off, L))
                rec(grp, off + L)

        rec(list(range(n)), 0)
        if len(segs) > self.max_segs:
            return False
        # keys per work item: the largest candidate that still gives every CTA of the
        # persistent grid ~4 items (long items amortise per-item costs; too few of them leave
        # SMs idle), read by the kernels from a device scalar so captured graphs follow it
        cands = [c for c in (1024, 512, 256, 128) if c <= self.chunk] or [self.chunk]
        chunk = cands[-1]
        for c in cands:
            if sum(max(1, -(-x[4] // c)) for x in segs) * self.Hkv >= self.target_items:
                chunk = c
                break
        rows = np.full((self.max_segs, self.SEG_STRIDE), -1, np.int32)
        slot = np.zeros((self.max_segs, self.SEG_STRIDE), np.int32)
        nslot = np.zeros(self.max_batch, np.int32)
        items = []
        for s, (rr, _, _, _, mx) in enumerate(segs):
            nch = max(1, -(-mx // chunk))
            if nch > 255:
                return False
            for j, b in enumerate(rr):
                rows[s, j] = b
                slot[s, j] = nslot[b]
                nslot[b] += nch
            items += [((s << 8) | c, min(chunk, mx - c * chunk)) for c in range(nch)]
        # longest items first: the persistent CTAs take items round-robin
        items = [it for it, _ in sorted(items, key=lambda x: -x[1])]
        if nslot.max(initial=0) > self.max_slots or len(items) > self.t_items.numel():
            return False
        k = len(segs)
        dev = self.t_rows.device
        self.t_rows.copy_(torch.from_numpy(rows.reshape(-1)).to(dev, non_blocking=False))
        self.t_slot.copy_(torch.from_numpy(slot.reshape(-1)).to(dev))
        self.t_start[:k].copy_(torch.tensor([x[1] for x in segs], dtype=torch.int32))
        self.t_len[:k].copy_(torch.tensor([x[2] for x in segs], dtype=torch.int32))
        self.t_off[:k].copy_(torch.tensor([x[3] for x in segs], dtype=torch.int32))
        self.t_items[:len(items)].copy_(torch.tensor(items, dtype=torch.int32))
        self.t_n.copy_(torch.tensor([len(items) * self.Hkv, chunk], dtype=torch.int32))
        self.t_nslot.copy_(torch.from_numpy(nslot).to(dev))
        self.stats = {"segments": k, "shared_segments": sum(1 for x in segs if x[2] >= 0), "items": len(items),
                      "max_slots": int(nslot.max(initial=0)), "chunk": chunk}
        return True

    def __call__(self, q, k_cache, v_cache, kv_indices, kv_len, out=None, scale=None):
        B = q.shape[0]
        if out is None:
            out = torch.empty(B, self.Hq * self.D, dtype=q.dtype, device=q.device)
        scale = scale if scale is not None else self.D ** -0.5
        ext().attn_decode_shared(q, k_cache, v_cache, kv_indices, kv_len.to(torch.int32), self.t_rows, self.t_slot,
                                 self.t_start, self.t_len, self.t_off, self.t_items, self.t_n, self.t_nslot, out,
                                 self.part_o, self.part_lse, self.Hq, self.Hkv, self.max_slots, self.chunk, scale,
                                 self.use_tc)
        return out
