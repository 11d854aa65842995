"""Inference-only op wrappers (no autograd) used by the rollout engine.

CUDA tensors call the sm_100a kernels directly; CPU tensors run the references, so the
engine's cursor / mount / radix logic is testable on a machine without a GPU.
"""
from __future__ import annotations

import torch

from . import reference as ref
from ._ext import ext
from .core import _rope_inplace


def rms(x, w, eps, plus_one=False):
    if x.is_cuda:
        return ext().rmsnorm_fwd(x, w, eps, plus_one)[0]
    return ref.rmsnorm(x, w, eps, plus_one).to(x.dtype)


def rope_(qkv, pos, Hq, Hkv, D, theta):
    _rope_inplace(qkv, pos, Hq, Hkv, D, theta, inverse=False)


def kv_write(qkv, Hq, Hkv, D, slots, kc, vc):
    if qkv.is_cuda:
        ext().kv_write(qkv, Hq, Hkv, D, slots, kc, vc)
        return
    w = Hkv * D
    ok = slots >= 0
    s = slots[ok]
    kc[s] = qkv[ok, Hq * D: Hq * D + w].to(kc.dtype)
    vc[s] = qkv[ok, Hq * D + w: Hq * D + 2 * w].to(vc.dtype)


def prefill_attn(q, kc, vc, plan, Hq, Hkv, D, scale):
    """q [T, Hq*D] against cache rows plan.key_idx (slot ids), bottom-right causal."""
    if q.is_cuda:
        from .core import use_tc_attention
        mode = use_tc_attention(D)
        o, _ = ext().attn_fwd(q, kc, vc, plan.cu_q, plan.cu_k, plan.key_idx, plan.tiles_for(mode), Hq, Hkv, D, scale,
                              True, False, mode)
        return o
    T = q.shape[0]
    o, _ = ref.gather_attention(q.reshape(T, Hq, D), kc.reshape(-1, Hkv, D), vc.reshape(-1, Hkv, D),
                                plan.host_cu_q, plan.host_cu_k, torch.from_numpy(plan.host_key_idx), scale)
    return o.reshape(T, Hq * D).to(q.dtype)


def gemm_res_norm(a, w, residual, norm_w, eps, plus_one=False, bias=None):
    """(x, h) = (a w^T + bias + residual, RMSNorm(x) * norm_w): on CUDA one split-K GEMM plus
    one finish kernel for decode-sized rows."""
    if a.is_cuda:
        x, h = ext().gemm_res_norm(a, w, residual, norm_w, eps, plus_one, bias)
        return x, h
    from .core import gemm
    x = gemm(a, w, bias=bias, residual=residual).to(residual.dtype)
    return x, rms(x, norm_w, eps, plus_one)


def qkv_rope_kv(h, w, bias, pos, theta, Hq, Hkv, D, slots, kc, vc):
    """q rows of h w^T + bias after the rotary embedding; the k / v rows go to the cache at
    `slots` (one GEMM + one finish kernel on CUDA for decode-sized rows)."""
    if h.is_cuda:
        return ext().gemm_qkv_rope(h, w, bias, pos, theta, Hq, Hkv, D, slots, kc, vc)
    from .core import gemm
    qkv = gemm(h, w, bias=bias).to(h.dtype)
    rope_(qkv, pos, Hq, Hkv, D, theta)
    kv_write(qkv, Hq, Hkv, D, slots, kc, vc)
    return qkv[:, : Hq * D]


def swiglu(gu):
    if gu.is_cuda:
        return ext().swiglu_fwd(gu)
    return ref.swiglu(gu).to(gu.dtype)


def embed(ids, W):
    if W.is_cuda:
        return ext().embed_fwd(ids, W)
    return W[ids]
