"""Autograd-aware ops over the sm_100a kernels, with CPU reference fallbacks.

Every op dispatches on the device of its input: CUDA tensors run the hand-written
kernels of ``octopus_b200._C`` (and raise if the extension is missing), CPU tensors
run :mod:`octopus_b200.ops.reference` in fp32/fp64 so the whole stack is testable on a
machine without a GPU.

Weight gradients: a weight tensor may carry an fp32 ``main_grad`` attribute (the
FSDP / optimizer gradient buffer).  Backward then accumulates straight into it (the
wgrad GEMM epilogue adds into fp32) and returns no gradient for the weight, so no
bf16 gradient tensor is ever materialised.

Reference parity: `octopus/rl/lm_head.py:20-153` (chunked head: per-row logprob and
entropy, recomputed in backward), `octopus/rl/prefix_tree.py:381-413` (tree attention:
bottom-right causal attention over gathered key lists), `octopus/rl/seq_tiles.py:61-82`
(rms_norm, silu_mul element-wise blocks).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

from . import reference as ref
from ._ext import ext

HEAD_CHUNK = 4096  # rows per chunk in the head backward (dz is [chunk, vocab] bf16)
CPU_VOCAB_CHUNK = 1024  # vocab columns per chunk of the CPU head (online log-sum-exp merge)


def use_tc_attention(D: int) -> int:
    """Attention forward kernel: 2 = tcgen05/TMEM with two query tiles per CTA (head_dim
    128: every BASELINE model), 0 = the mma.sync kernel for other head dims (the tiny
    test models use 64)."""
    return 2 if D == 128 else 0


def use_tc_bwd(D: int) -> int:
    """Attention backward kernels: 1 = tcgen05/TMEM (head_dim 128), 0 = mma.sync (other
    head dims)."""
    return int(D == 128)


def _is_cuda(t: torch.Tensor) -> bool:
    return t.is_cuda


def _accum_wgrad(w: torch.Tensor, dw: torch.Tensor):
    """Accumulate a weight gradient into w.main_grad if present, else return it."""
    mg = getattr(w, "main_grad", None)
    if mg is not None:
        mg.add_(dw.to(mg.dtype).view_as(mg))
        return None
    return dw.to(w.dtype)


# ---------------------------------------------------------------------------- GEMM
def gemm(a: torch.Tensor, b: torch.Tensor, *, a_mn: bool = False, b_mn: bool = False, out=None,
         out_dtype=torch.bfloat16, alpha: float = 1.0, residual=None, bias=None, accumulate: bool = False,
         bn: int = 0) -> torch.Tensor:
    """C = alpha * A_log @ B_log^T (+bias)(+residual) on the tcgen05 GEMM.

    A_log is `a` ([M, K]) or `a.T` when a_mn ([K, M] storage); B_log is `b` ([N, K]) or
    `b.T` when b_mn ([K, N] storage).
    """
    M = a.shape[1] if a_mn else a.shape[0]
    N = b.shape[1] if b_mn else b.shape[0]
    if not _is_cuda(a):
        A = a.t() if a_mn else a
        B = b.t() if b_mn else b
        y = alpha * (ref._f(A) @ ref._f(B).t())
        if bias is not None:
            y = y + ref._f(bias)
        if residual is not None:
            y = y + ref._f(residual)
        if out is not None:
            if accumulate:
                out.add_(y.to(out.dtype))
            else:
                out.copy_(y.to(out.dtype))
            return out
        return y.to(a.dtype if a.dtype in (torch.float32, torch.float64) else out_dtype)
    K = a.shape[0] if a_mn else a.shape[1]
    if M % 8 or N % 8 or K % 8:
        # the tcgen05 GEMM's granularity; checked here so the extension never sees such a shape
        raise ValueError(f"gemm: M, N, K must be multiples of 8 on the GPU (got {M}, {N}, {K})")
    if out is None:
        out = torch.empty(M, N, dtype=out_dtype, device=a.device)
    ext().gemm_out(a, a_mn, b, b_mn, out, alpha, residual, bias, accumulate, bn)
    return out


class _Linear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, b, residual):
        ctx.save_for_backward(x, w)
        ctx.bias = b
        ctx.has_res = residual is not None
        if _is_cuda(x):
            return gemm(x, w, bias=b, residual=residual)
        return ref.linear(x, w, b, residual).to(x.dtype)

    @staticmethod
    def backward(ctx, dy):
        x, w = ctx.saved_tensors
        dy = dy.contiguous()
        dres = dy if ctx.has_res else None
        dx, dw, db = _linear_grads(x, w, ctx.bias, dy, ctx.needs_input_grad[1])
        return dx, dw, db, dres


def _linear_grads(x, w, bias, dy, w_needs_grad):
    """(dx, dw, db) of y = x W^T + b: the weight gradient accumulates into W.main_grad (fp32)
    when W has one (then dw is None), the bias gradient likewise."""
    db = None
    if bias is not None:
        db = _accum_wgrad(bias, dy.float().sum(0) if dy.dtype != torch.float64 else dy.sum(0))
    mg = getattr(w, "main_grad", None)
    frozen = mg is None and not w_needs_grad  # (LoRA base weights: no weight gradient)
    if _is_cuda(x):
        dx = gemm(dy, w, b_mn=True)  # dy [M,N] @ w [N,K]
        if frozen:
            dw = None
        elif mg is not None:
            gemm(dy, x, a_mn=True, b_mn=True, out=mg, accumulate=True)
            dw = None
        else:
            dw = gemm(dy, x, a_mn=True, b_mn=True, out_dtype=torch.float32).to(w.dtype)
    else:
        dx = (ref._f(dy) @ ref._f(w)).to(x.dtype)
        dw = None if frozen else _accum_wgrad(w, ref._f(dy).t() @ ref._f(x))
    return dx, dw, db


def linear(x, w, b=None, residual=None, lora=None):
    """y = x W^T (+ b) (+ residual) with fused fp32 weight-gradient accumulation; with
    lora = (A [r, in], B [out, r], scale) the adapter term scale * (x A^T) B^T is added."""
    if lora is not None:
        return _LoraLinear.apply(x, w, b, residual, lora[0], lora[1], float(lora[2]))
    return _Linear.apply(x, w, b, residual)


class _LoraLinear(torch.autograd.Function):
    """Frozen base W plus a trained low-rank adapter:
        u = x A^T [M, r];  y = x W^T (+ b) (+ residual) + s u B^T
    backward (base W gets no gradient):
        du = s dy B;  dB += s dy^T u;  dA += du^T x;  dx = dy W + du A
    Adapter gradients accumulate into A.main_grad / B.main_grad (fp32)."""

    @staticmethod
    def forward(ctx, x, w, b, residual, A, B, s):
        ctx.s = s
        ctx.has_res, ctx.bias = residual is not None, b
        u = gemm(x, A)
        v = gemm(u, B, alpha=s, residual=residual)
        y = gemm(x, w, bias=b, residual=v)
        ctx.save_for_backward(x, w, A, B, u)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w, A, B, u = ctx.saved_tensors
        s = ctx.s
        dy = dy.contiguous()
        db = None
        if ctx.bias is not None and ctx.needs_input_grad[2]:
            db = _accum_wgrad(ctx.bias, dy.float().sum(0) if dy.dtype != torch.float64 else dy.sum(0))
        du = gemm(dy, B, b_mn=True, alpha=s)               # [M, r]
        gB = getattr(B, "main_grad", None)
        gA = getattr(A, "main_grad", None)
        if gB is not None:
            gemm(dy, u, a_mn=True, b_mn=True, alpha=s, out=gB, accumulate=True)
        if gA is not None:
            gemm(du, x, a_mn=True, b_mn=True, out=gA, accumulate=True)
        dx = gemm(dy, w, b_mn=True, residual=gemm(du, A, b_mn=True))
        return dx, None, db, (dy if ctx.has_res else None), None, None, None


# ---------------------------------------------------------------------------- RMSNorm
class _RMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, eps, plus_one):
        ctx.eps, ctx.plus_one = eps, plus_one
        if _is_cuda(x):
            y, rstd = ext().rmsnorm_fwd(x, w, eps, plus_one)
        else:
            xf = ref._f(x)
            rstd = torch.rsqrt(xf.pow(2).mean(-1) + eps)
            y = ref.rmsnorm(x, w, eps, plus_one).to(x.dtype)
        ctx.save_for_backward(x, w, rstd)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w, rstd = ctx.saved_tensors
        dy = dy.contiguous()
        if _is_cuda(x):
            mg = getattr(w, "main_grad", None)
            dwbuf = mg if mg is not None else torch.zeros(w.shape, dtype=torch.float32, device=w.device)
            dx = ext().rmsnorm_bwd(dy, x, w, rstd, None, dwbuf, ctx.plus_one)
            dw = None if mg is not None else dwbuf.to(w.dtype)
            return dx, dw, None, None
        xf, dyf, wf = ref._f(x), ref._f(dy), ref._f(w)
        weff = (1.0 + wf) if ctx.plus_one else wf
        r = rstd[:, None]
        xh = xf * r
        gw = dyf * weff
        dx = r * (gw - xh * (gw * xh).mean(-1, keepdim=True))
        dw = _accum_wgrad(w, (dyf * xh).sum(0))
        return dx.to(x.dtype), dw, None, None


def rmsnorm(x, w, eps: float = 1e-6, plus_one: bool = False):
    return _RMSNorm.apply(x, w, eps, plus_one)


# ---------------------------------------------------------------------------- RoPE
class _Rope(torch.autograd.Function):
    """In-place rotary embedding on the q and k heads of a fused qkv row."""

    @staticmethod
    def forward(ctx, qkv, pos, Hq, Hkv, D, theta):
        ctx.meta = (Hq, Hkv, D, theta)
        ctx.save_for_backward(pos)
        _rope_inplace(qkv, pos, Hq, Hkv, D, theta, inverse=False)
        ctx.mark_dirty(qkv)
        return qkv

    @staticmethod
    def backward(ctx, g):
        (pos,) = ctx.saved_tensors
        Hq, Hkv, D, theta = ctx.meta
        g = g.contiguous().clone()
        _rope_inplace(g, pos, Hq, Hkv, D, theta, inverse=True)
        return g, None, None, None, None, None


def _rope_inplace(qkv, pos, Hq, Hkv, D, theta, inverse):
    if _is_cuda(qkv):
        ext().rope(qkv, pos, Hq, Hkv, D, theta, inverse)
        return
    T = qkv.shape[0]
    heads = qkv[:, : (Hq + Hkv) * D].reshape(T, Hq + Hkv, D)
    heads.copy_(ref.rope(heads, pos, theta, inverse=inverse).to(qkv.dtype))


def rope_(qkv, pos, Hq, Hkv, D, theta):
    return _Rope.apply(qkv, pos, Hq, Hkv, D, theta)


class _LinearRope(torch.autograd.Function):
    """qkv = rope(x W^T + b) in one tcgen05 GEMM (the rotary embedding in its epilogue);
    backward: the inverse rotation of the gradient, then the linear layer's gradients."""

    @staticmethod
    def forward(ctx, x, w, b, pos, Hq, Hkv, D, theta):
        ctx.meta = (Hq, Hkv, D, theta)
        ctx.bias = b
        ctx.save_for_backward(x, w, pos)
        return ext().gemm_rope(x, w, b, pos, theta, Hq, Hkv, D)

    @staticmethod
    def backward(ctx, dy):
        x, w, pos = ctx.saved_tensors
        Hq, Hkv, D, theta = ctx.meta
        g = dy.contiguous().clone()
        _rope_inplace(g, pos, Hq, Hkv, D, theta, inverse=True)
        dx, dw, db = _linear_grads(x, w, ctx.bias, g, ctx.needs_input_grad[1])
        return dx, dw, db, None, None, None, None, None


def linear_rope(x, w, b, pos, Hq, Hkv, D, theta):
    """rope(x W^T + b) on the q / k heads of the fused qkv projection: one GEMM with the
    rotation in its epilogue on CUDA (head_dim 64 / 128), else linear then rope_."""
    if (_is_cuda(x) and D in (64, 128) and x.shape[0] % 8 == 0 and x.shape[1] % 8 == 0 and x.stride(1) == 1
            and w.stride(1) == 1 and pos.dtype == torch.int32):
        return _LinearRope.apply(x, w, b, pos.contiguous(), Hq, Hkv, D, theta)
    return rope_(linear(x, w, b), pos, Hq, Hkv, D, theta)


# ---------------------------------------------------------------------------- SwiGLU
class _SwiGLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gu):
        ctx.save_for_backward(gu)
        if _is_cuda(gu):
            return ext().swiglu_fwd(gu)
        return ref.swiglu(gu).to(gu.dtype)

    @staticmethod
    def backward(ctx, d):
        (gu,) = ctx.saved_tensors
        d = d.contiguous()
        if _is_cuda(gu):
            return ext().swiglu_bwd(gu, d)
        g, u = ref._f(gu).chunk(2, dim=-1)
        s = torch.sigmoid(g)
        df = ref._f(d)
        return torch.cat([df * u * s * (1 + g * (1 - s)), df * g * s], dim=-1).to(gu.dtype)


def swiglu(gu):
    return _SwiGLU.apply(gu)


def gemm_swiglu_ok(x, gu_w) -> bool:
    """Whether gemm_swiglu runs as one fused GEMM for these operands."""
    return (_is_cuda(x) and x.dim() == 2 and gu_w.shape[0] % 256 == 0 and x.shape[0] % 8 == 0
            and x.shape[1] % 8 == 0 and x.stride(1) == 1 and gu_w.stride(1) == 1)


def gemm_swiglu(x, gu_w):
    """swiglu(x gu_w^T) with gu_w = [W_gate; W_up] ([2F, K]), forward only (no autograd).

    On CUDA (F a multiple of 128) one tcgen05 GEMM pairs each 128-row gate tile with its
    up tile and applies silu(gate) * up in the epilogue: the [M, 2F] projection is never
    written.  The result equals the unfused GEMM + swiglu (gate and up rounded to bf16
    before the activation).  Otherwise: the GEMM, then swiglu."""
    if gemm_swiglu_ok(x, gu_w):
        return ext().gemm_swiglu(x, gu_w)
    if _is_cuda(x):
        return ext().swiglu_fwd(gemm(x, gu_w))
    return ref.swiglu(ref.linear(x, gu_w, None, None).to(x.dtype)).to(x.dtype)


# ---------------------------------------------------------------------------- embedding
class _Embed(torch.autograd.Function):
    # `anchor` (an empty tensor that requires grad) records the op in the graph when the
    # table itself does not require grad: its gradient goes to W.main_grad
    @staticmethod
    def forward(ctx, ids, W, anchor):
        ctx.save_for_backward(ids, W)
        if _is_cuda(W):
            return ext().embed_fwd(ids, W)
        return W[ids]

    @staticmethod
    def backward(ctx, d):
        ids, W = ctx.saved_tensors
        d = d.contiguous()
        mg = getattr(W, "main_grad", None)
        if _is_cuda(W):
            buf = mg if mg is not None else torch.zeros(W.shape, dtype=torch.float32, device=W.device)
            ext().embed_bwd(ids, d, buf)
            return None, (None if mg is not None or not W.requires_grad else buf.to(W.dtype)), None
        g = torch.zeros(W.shape, dtype=ref._f(d).dtype)
        g.index_add_(0, ids, ref._f(d))
        wg = _accum_wgrad(W, g)
        return None, (wg if W.requires_grad else None), None


def embed(ids, W):
    """Rows W[ids]; under grad mode the table's gradient accumulates into W.main_grad."""
    anchor = None
    if torch.is_grad_enabled() and not W.requires_grad and hasattr(W, "main_grad"):
        anchor = torch.empty(0, device=W.device, requires_grad=True)
    return _Embed.apply(ids, W, anchor)


# ---------------------------------------------------------------------------- attention plan
@dataclass
class AttnPlan:
    """Sequences of query rows with gathered key lists (tree nodes or requests).

    cu_q[s]..cu_q[s+1] are the query rows of sequence s; key_idx[cu_k[s]..cu_k[s+1]]
    its key rows (own rows last).  Tile tables are precomputed on the host.
    """

    cu_q: torch.Tensor
    cu_k: torch.Tensor
    key_idx: torch.Tensor
    fwd_tiles: torch.Tensor
    dq_tiles: torch.Tensor
    kv_tiles: torch.Tensor
    fwd_tiles_pp: torch.Tensor  # 256-row query tiles, most keys first (two-tile tcgen05 forward)
    dq_tiles_tc: torch.Tensor   # 128-row query tiles, most keys first (tcgen05 backward)
    kv_tiles_tc: torch.Tensor   # 128-row key tiles of sequences with queries, most work first
    host_cu_q: np.ndarray = field(repr=False, default=None)
    host_cu_k: np.ndarray = field(repr=False, default=None)
    host_key_idx: np.ndarray = field(repr=False, default=None)

    @staticmethod
    def build(cu_q, cu_k, key_idx, device="cpu") -> "AttnPlan":
        cu_q = np.asarray(cu_q, dtype=np.int32)
        cu_k = np.asarray(cu_k, dtype=np.int32)
        key_idx = np.asarray(key_idx, dtype=np.int32)
        nq = np.diff(cu_q)
        nk = np.diff(cu_k)

        def tiles(lengths, step, mask):
            out = []
            for s, n in enumerate(lengths):
                if n <= 0 or not mask[s]:
                    continue
                for o in range(0, int(n), step):
                    out.append((s, o))
            return np.asarray(out, dtype=np.int32).reshape(-1, 2)

        has_q = nq > 0
        ft = tiles(nq, 128, has_q)
        pp = tiles(nq, 256, has_q)
        if len(pp):
            # longest CTAs first: keys visible to the tile's last row (bottom-right causal)
            s_, q0 = pp[:, 0], pp[:, 1]
            rows = np.minimum(256, nq[s_] - q0)
            work = np.minimum(nk[s_], q0 + rows + nk[s_] - nq[s_]) * rows
            pp = pp[np.argsort(-work, kind="stable")]
        dqt = tiles(nq, 128, has_q)
        if len(dqt):
            s_, q0 = dqt[:, 0], dqt[:, 1]
            rows = np.minimum(128, nq[s_] - q0)
            dqt = dqt[np.argsort(-(np.minimum(nk[s_], q0 + rows + nk[s_] - nq[s_]) * rows), kind="stable")]
        kvt = tiles(nk, 128, has_q)
        if len(kvt):
            # queries that see key tile k0: those from max(0, k0 - (nk - nq)) on
            s_, k0 = kvt[:, 0], kvt[:, 1]
            seen = nq[s_] - np.clip(k0 - (nk[s_] - nq[s_]), 0, nq[s_])
            kvt = kvt[np.argsort(-(seen * np.minimum(128, nk[s_] - k0)), kind="stable")]
        dt = tiles(nq, 64, has_q)
        kt = tiles(nk, 64, has_q)
        dev = torch.device(device)
        from ..utils.iostats import h2d

        def T(a):
            return h2d(np.ascontiguousarray(a), dev)

        return AttnPlan(T(cu_q), T(cu_k), T(key_idx), T(ft.reshape(-1)), T(dt.reshape(-1)), T(kt.reshape(-1)),
                        T(pp.reshape(-1)), T(dqt.reshape(-1)), T(kvt.reshape(-1)), cu_q, cu_k, key_idx)

    def tiles_for(self, mode: int) -> torch.Tensor:
        """Forward tile table of attention kernel `mode` (see use_tc_attention)."""
        return self.fwd_tiles_pp if mode == 2 else self.fwd_tiles

    @staticmethod
    def causal_packed(lengths, device="cpu") -> "AttnPlan":
        """Plain packed causal sequences (keys = own rows)."""
        cu = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
        return AttnPlan.build(cu, cu, np.arange(cu[-1], dtype=np.int32), device)


class _Attention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, plan, Hq, Hkv, D, scale):
        T, W = qkv.shape
        q = qkv[:, : Hq * D]
        k = qkv[:, Hq * D: (Hq + Hkv) * D]
        v = qkv[:, (Hq + Hkv) * D: (Hq + 2 * Hkv) * D]
        ctx.meta = (plan, Hq, Hkv, D, scale)
        if _is_cuda(qkv):
            mode = use_tc_attention(D)
            o, lse = ext().attn_fwd(q, k, v, plan.cu_q, plan.cu_k, plan.key_idx, plan.tiles_for(mode), Hq, Hkv, D,
                                    scale, True, True, mode)
        else:
            o3, lse = ref.gather_attention(q.reshape(T, Hq, D), k.reshape(T, Hkv, D), v.reshape(T, Hkv, D),
                                           plan.host_cu_q, plan.host_cu_k, torch.from_numpy(plan.host_key_idx),
                                           scale)
            o = o3.reshape(T, Hq * D).to(qkv.dtype)
        ctx.save_for_backward(qkv, o, lse)
        return o

    @staticmethod
    def backward(ctx, do):
        qkv, o, lse = ctx.saved_tensors
        plan, Hq, Hkv, D, scale = ctx.meta
        T = qkv.shape[0]
        do = do.contiguous()
        if _is_cuda(qkv):
            q = qkv[:, : Hq * D]
            k = qkv[:, Hq * D: (Hq + Hkv) * D]
            v = qkv[:, (Hq + Hkv) * D: (Hq + 2 * Hkv) * D]
            dk = torch.zeros(T, Hkv * D, dtype=torch.float32, device=qkv.device)
            dv = torch.zeros(T, Hkv * D, dtype=torch.float32, device=qkv.device)
            tc = use_tc_bwd(D)
            dq = ext().attn_bwd(q, k, v, o, do, lse, plan.cu_q, plan.cu_k, plan.key_idx,
                                plan.dq_tiles_tc if tc else plan.dq_tiles, plan.kv_tiles_tc if tc else plan.kv_tiles,
                                dk, dv, Hq, Hkv, D, scale, True, tc)
            dqkv = torch.empty_like(qkv)
            dqkv[:, : Hq * D] = dq
            dqkv[:, Hq * D: (Hq + Hkv) * D] = dk
            dqkv[:, (Hq + Hkv) * D:] = dv
            return dqkv, None, None, None, None, None
        # CPU: differentiate the reference with autograd
        with torch.enable_grad():
            x = qkv.detach().to(torch.float64 if qkv.dtype == torch.float64 else torch.float32).requires_grad_(True)
            q = x[:, : Hq * D].reshape(T, Hq, D)
            k = x[:, Hq * D: (Hq + Hkv) * D].reshape(T, Hkv, D)
            v = x[:, (Hq + Hkv) * D:].reshape(T, Hkv, D)
            o3, _ = ref.gather_attention(q, k, v, plan.host_cu_q, plan.host_cu_k,
                                         torch.from_numpy(plan.host_key_idx), scale)
            (g,) = torch.autograd.grad(o3.reshape(T, Hq * D), x, ref._f(do).to(x.dtype))
        return g.to(qkv.dtype), None, None, None, None, None


class _AttentionKV(torch.autograd.Function):
    """Gathered-key attention with separate q [Tq, Hq*D] and k, v [rows, Hkv*D]: the key
    rows may extend past the query rows (chunk-major training appends the kept k / v of
    earlier chunks after a chunk's own rows)."""

    @staticmethod
    def forward(ctx, q, k, v, plan, Hq, Hkv, D, scale):
        ctx.meta = (plan, Hq, Hkv, D, scale)
        if _is_cuda(q):
            mode = use_tc_attention(D)
            o, lse = ext().attn_fwd(q, k, v, plan.cu_q, plan.cu_k, plan.key_idx, plan.tiles_for(mode), Hq, Hkv, D,
                                    scale, True, True, mode)
            ctx.save_for_backward(q, k, v, o, lse)
            return o
        o3, _ = ref.gather_attention(q.reshape(q.shape[0], Hq, D), k.reshape(k.shape[0], Hkv, D),
                                     v.reshape(v.shape[0], Hkv, D), plan.host_cu_q, plan.host_cu_k,
                                     torch.from_numpy(plan.host_key_idx), scale)
        ctx.save_for_backward(q, k, v)
        return o3.reshape(q.shape[0], Hq * D).to(q.dtype)

    @staticmethod
    def backward(ctx, do):
        plan, Hq, Hkv, D, scale = ctx.meta
        do = do.contiguous()
        if _is_cuda(do):
            q, k, v, o, lse = ctx.saved_tensors
            dk = torch.zeros(k.shape[0], Hkv * D, dtype=torch.float32, device=k.device)
            dv = torch.zeros_like(dk)
            tc = use_tc_bwd(D)
            dq = ext().attn_bwd(q, k, v, o, do, lse, plan.cu_q, plan.cu_k, plan.key_idx,
                                plan.dq_tiles_tc if tc else plan.dq_tiles, plan.kv_tiles_tc if tc else plan.kv_tiles,
                                dk, dv, Hq, Hkv, D, scale, True, tc)
            return dq, dk.to(k.dtype), dv.to(v.dtype), None, None, None, None, None
        q, k, v = ctx.saved_tensors
        with torch.enable_grad():
            ins = [t.detach().requires_grad_(True) for t in (q, k, v)]
            o3, _ = ref.gather_attention(ins[0].reshape(q.shape[0], Hq, D), ins[1].reshape(k.shape[0], Hkv, D),
                                         ins[2].reshape(v.shape[0], Hkv, D), plan.host_cu_q, plan.host_cu_k,
                                         torch.from_numpy(plan.host_key_idx), scale)
            g = torch.autograd.grad(o3.reshape(q.shape[0], Hq * D), ins, ref._f(do).to(o3.dtype))
        return g[0].to(q.dtype), g[1].to(k.dtype), g[2].to(v.dtype), None, None, None, None, None


def attention_kv(q, k, v, plan: AttnPlan, Hq: int, Hkv: int, D: int, scale: float | None = None):
    """Gathered-key causal attention of q rows against k / v rows (key_idx indexes k / v)."""
    if scale is None:
        scale = D ** -0.5
    return _AttentionKV.apply(q, k, v, plan, Hq, Hkv, D, scale)


def attention(qkv, plan: AttnPlan, Hq: int, Hkv: int, D: int, scale: float | None = None):
    """Gathered-key causal attention on a fused qkv [T, (Hq+2Hkv)*D] -> o [T, Hq*D]."""
    if scale is None:
        scale = D ** -0.5
    return _Attention.apply(qkv, plan, Hq, Hkv, D, scale)


# ---------------------------------------------------------------------------- logprob head
class _Head(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, W, labels, alpha, vocab_limit):
        M = h.shape[0]
        ctx.alpha, ctx.vocab_limit = alpha, vocab_limit
        if M == 0:  # no trained pair (an empty micro-batch that keeps the ranks' collectives paired)
            z = torch.zeros(0, dtype=torch.float32, device=h.device)
            ctx.save_for_backward(h, W, labels, z, z)
            return z, z.clone()
        if _is_cuda(h):
            pad = (-M) % 8
            hp = torch.cat([h, h.new_zeros(pad, h.shape[1])]) if pad else h
            lp = torch.cat([labels, labels.new_full((pad,), -1)]) if pad else labels
            logp, ent, lse = ext().head_fwd(hp.contiguous(), W, lp.to(torch.int32).contiguous(), alpha,
                                            vocab_limit or 0)
            logp, ent, lse = logp[:M], ent[:M], lse[:M]
        else:
            logp, ent, lse = ref.logprob_head(h, W, labels, alpha, vocab_limit, vocab_chunk=CPU_VOCAB_CHUNK)
        ctx.save_for_backward(h, W, labels, lse, ent)
        return logp, ent

    @staticmethod
    def backward(ctx, g_lp, g_ent):
        h, W, labels, lse, ent = ctx.saved_tensors
        alpha, vocab_limit = ctx.alpha, ctx.vocab_limit
        M = h.shape[0]
        if g_lp is None:
            g_lp = torch.zeros_like(lse)
        if g_ent is None:
            g_ent = torch.zeros_like(lse)
        g_lp = g_lp.float().contiguous()
        g_ent = g_ent.float().contiguous()
        mg = getattr(W, "main_grad", None)
        frozen = mg is None and not ctx.needs_input_grad[1]
        if M == 0:
            return torch.zeros_like(h), (None if (mg is not None or frozen) else torch.zeros_like(W)), None, None, None
        if _is_cuda(h):
            dh = torch.empty_like(h)
            dW = mg if mg is not None else (None if frozen else
                                             torch.zeros(W.shape, dtype=torch.float32, device=W.device))
            V = W.shape[0]
            for a in range(0, M, HEAD_CHUNK):
                b = min(M, a + HEAD_CHUNK)
                m = b - a
                pad = (-m) % 8
                hc = h[a:b]
                lc, sc, ec, gl, ge = labels[a:b], lse[a:b], ent[a:b], g_lp[a:b], g_ent[a:b]
                if pad:
                    hc = torch.cat([hc, hc.new_zeros(pad, hc.shape[1])])
                    lc = torch.cat([lc, lc.new_full((pad,), -1)])
                    z = torch.zeros(pad, dtype=torch.float32, device=h.device)
                    sc, ec, gl, ge = (torch.cat([t, z]) for t in (sc, ec, gl, ge))
                hc = hc.contiguous()
                dz = torch.empty(hc.shape[0], V, dtype=torch.bfloat16, device=h.device)
                ext().head_grad_logits(hc, W, lc.to(torch.int32).contiguous(), sc.contiguous(), ec.contiguous(),
                                       gl.contiguous(), ge.contiguous(), dz, alpha, vocab_limit or 0)
                dh[a:b] = gemm(dz, W, b_mn=True)[:m]
                if dW is not None:
                    gemm(dz, hc, a_mn=True, b_mn=True, out=dW, accumulate=True)
            dWret = None if (mg is not None or dW is None) else dW.to(W.dtype)
            return dh, dWret, None, None, None
        with torch.enable_grad():
            hf = ref._f(h).detach().requires_grad_(True)
            Wf = ref._f(W).detach().requires_grad_(True)
            lp, en, _ = ref.logprob_head(hf, Wf, labels, alpha, vocab_limit)
            gh, gW = torch.autograd.grad((lp * g_lp.to(lp.dtype)).sum() + (en * g_ent.to(en.dtype)).sum(),
                                         (hf, Wf))
        return gh.to(h.dtype), _accum_wgrad(W, gW), None, None, None


def logprob_head(h, W, labels, alpha: float = 1.0, vocab_limit: int | None = None):
    """(log p(label), entropy) of softmax(alpha * h W^T) without full logits."""
    return _Head.apply(h, W, labels, alpha, vocab_limit)


# ---------------------------------------------------------------------------- sampling
def _lowbias32(x: torch.Tensor) -> torch.Tensor:
    """Wellons' "lowbias32" 32-bit integer finaliser on int64 tensors holding 32-bit values."""
    M32 = 0xFFFFFFFF
    x = x ^ (x >> 16)
    x = (x * 0x7FEB352D) & M32
    x = x ^ (x >> 15)
    x = (x * 0x846CA68B) & M32
    return x ^ (x >> 16)


def _uniform(seed: int, stream: torch.Tensor, V: int) -> torch.Tensor:
    """Counter-based uniforms in (0, 1), [rows, V]: a 32-bit integer hash of (seed, row
    stream, token), so a row's draws do not depend on the batch.  All 64 bits of the
    stream (request id << 32 | position) enter the row key."""
    M32 = 0xFFFFFFFF
    s = stream.to(torch.int64)
    lo, hi = s & M32, (s >> 32) & M32
    key = _lowbias32(((hi * 0x9E3779B1) & M32) ^ ((int(seed) & M32) * 0x85EBCA77 & M32))
    key = _lowbias32(((lo * 0x27D4EB2F) & M32) ^ key)
    tok = torch.arange(V, device=stream.device, dtype=torch.int64)
    x = _lowbias32((key[:, None] ^ ((tok[None, :] * 0xC2B2AE3D) & M32)) & M32)
    return (x.to(torch.float64) + 0.5) / 4294967296.0


def filter_logits(z: torch.Tensor, top_p: float = 1.0, top_k: int = 0) -> torch.Tensor:
    """Mask of the tokens kept by top-k (k <= 0 or k >= vocab: no top-k), then top-p on the
    renormalised distribution (the smallest set of highest-probability tokens whose mass
    reaches p; the top token is always kept)."""
    V = z.shape[-1]
    keep = torch.ones_like(z, dtype=torch.bool)
    if 0 < top_k < V:
        kth = z.topk(int(top_k), dim=-1).values[:, -1:]
        keep &= z >= kth
    if top_p < 1.0:
        zs, idx = z.masked_fill(~keep, float("-inf")).sort(dim=-1, descending=True)
        p = torch.softmax(zs, dim=-1)
        before = p.cumsum(-1) - p  # mass of the higher-ranked tokens
        drop = before >= top_p
        drop[:, 0] = False
        keep &= ~torch.zeros_like(drop).scatter(1, idx, drop)
    return keep


def _sample_filtered(h, W, alpha, seed, row_stream, vocab_limit, top_p, top_k):
    """Sampling with top-p / top-k: logits of the rows (one GEMM), the filter, Gumbel-max over
    the kept tokens.  The logprob is under the full tempered distribution (what the trainer
    recomputes)."""
    V = vocab_limit or W.shape[0]
    if _is_cuda(h):
        M = h.shape[0]
        pad = (-M) % 8
        hp = torch.cat([h, h.new_zeros(pad, h.shape[1])]) if pad else h
        z = gemm(hp.contiguous(), W, out_dtype=torch.float32)[:M, :V] * alpha
    else:
        z = (ref._f(h) @ ref._f(W).t())[:, :V] * alpha
    rs = row_stream if row_stream is not None else torch.arange(z.shape[0], device=z.device)
    toks, lps = [], []
    for a in range(0, z.shape[0], 32):  # row blocks bound the [rows, vocab] temporaries
        zb = z[a:a + 32]
        keep = filter_logits(zb, top_p, top_k)
        g = -torch.log(-torch.log(_uniform(seed, rs[a:a + 32], V))).to(zb.dtype)
        tok = (zb + g).masked_fill(~keep, float("-inf")).argmax(-1)
        toks.append(tok)
        lps.append(torch.log_softmax(zb, -1).gather(1, tok[:, None])[:, 0])
    return torch.cat(toks), torch.cat(lps).float()


def sample(h, W, temperature: float = 1.0, seed: int = 0, row_stream=None, vocab_limit: int | None = None,
           top_p: float = 1.0, top_k: int = 0):
    """Sample one token per row from softmax(h W^T / T) (Gumbel-max); returns (tokens, logprobs).
    With top_p < 1 or 0 < top_k < vocab the distribution is filtered first (_sample_filtered);
    otherwise the fused head samples without materialising logits."""
    alpha = 1.0 / max(temperature, 1e-6)
    V = vocab_limit or W.shape[0]
    if top_p < 1.0 or 0 < top_k < V:
        return _sample_filtered(h, W, alpha, seed, row_stream, vocab_limit, float(top_p), int(top_k))
    if _is_cuda(h):
        M = h.shape[0]
        pad = (-M) % 8
        hp = torch.cat([h, h.new_zeros(pad, h.shape[1])]) if pad else h
        rs = row_stream
        if rs is not None and pad:
            rs = torch.cat([rs, rs.new_zeros(pad)])
        tok, lp = ext().sample_head(hp.contiguous(), W, alpha, seed, rs, vocab_limit or 0)
        return tok[:M], lp[:M]
    z = (ref._f(h) @ ref._f(W).t()) * alpha
    if vocab_limit is not None:
        z = z[:, :vocab_limit]
    # counter-based noise of (seed, row stream, token): a row's sample does not depend on
    # which other rows share its batch (as on the GPU)
    rs = row_stream.cpu() if row_stream is not None else torch.arange(z.shape[0])
    u = _uniform(seed, rs, z.shape[1]).to(z.dtype)
    tok = (z - torch.log(-torch.log(u))).argmax(-1)
    lp = torch.log_softmax(z, -1).gather(1, tok[:, None])[:, 0]
    return tok, lp.float()


# ---------------------------------------------------------------------------- optimizer
def adamw_(p32, grad, m, v, p16, *, lr, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.0, step=1, sqnorm=None,
           max_norm=0.0, grad_scale=1.0):
    """Fused AdamW on flat fp32 buffers (+ bf16 copy), clip factor from a device-side norm."""
    if _is_cuda(p32):
        ext().adamw(p32, grad, m, v, p16, lr, betas[0], betas[1], eps, weight_decay, step, sqnorm, max_norm,
                    grad_scale)
        return
    b1, b2 = betas
    clip = grad_scale
    if sqnorm is not None and max_norm > 0:
        nrm = float(sqnorm.sqrt()) * grad_scale
        if nrm > max_norm:
            clip *= max_norm / (nrm + 1e-6)
    g = grad * clip
    m.mul_(b1).add_(g, alpha=1 - b1)
    v.mul_(b2).addcmul_(g, g, value=1 - b2)
    p32.mul_(1 - lr * weight_decay)
    bc1 = 1 - b1 ** step
    bc2 = 1 - b2 ** step
    p32.sub_(lr * (m / bc1) / ((v / bc2).sqrt() + eps))
    if p16 is not None:
        p16.copy_(p32.to(p16.dtype))


def sqnorm_(g: torch.Tensor, out: torch.Tensor):
    """out += sum(g^2) (device-side, no sync)."""
    if _is_cuda(g):
        ext().sqnorm_accum(g, out)
    else:
        out.add_(g.double().pow(2).sum().to(out.dtype))
