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
