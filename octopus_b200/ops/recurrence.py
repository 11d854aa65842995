"""Linear recurrences (gated delta rule / simple GLA) and the causal depthwise conv1d of
hybrid models, as autograd ops over variable-length segments with initial / final states.

CUDA tensors run the sm_100a kernels of csrc/recurrence.cu (or, with
OCTO_RECURRENCE_CHUNKED=1, the chunked tensor-op form); CPU tensors run the chunked form
(`recurrence_chunked`, autograd through its tensor ops).  `recurrence_ref` is the
token-by-token oracle (as in the reference's tests).

  recurrence(q, k, v, g, beta, segs, scale, delta, init_state, init_idx) -> (o, final)
      q, k, v [rows, H * d]; g, beta [rows, H] fp32; segs: host [(start, len)];
      init_state [n, H, d, d] fp32 with init_idx[s] its row for segment s (-1: zeros);
      final [n_seg, H, d, d] differentiable (a child segment's initial state).
  causal_conv(x, w, bias, segs, ctx, ctx_idx, silu) -> y
      x [rows, C]; w [C, W] fp32; ctx [n, W - 1, C] fp32 rows preceding each segment.

Reference parity (behaviour): the fla calls routed by `octopus/rl/gdn_varlen.py:18-36` and
`octopus/rl/mamba2_varlen.py`; the token-by-token references of `tests/test_chunk_major.py`.
"""
from __future__ import annotations

import numpy as np
import torch

from ._ext import ext


def _seg_tensor(segs, device):
    a = np.asarray(segs, dtype=np.int32).reshape(-1, 2).T.copy()
    return torch.from_numpy(a).to(device)


def _ckpt_offsets(segs, chunk):
    n = [(int(l) + chunk - 1) // chunk if int(l) > 0 else 0 for _, l in segs]
    off = np.concatenate([[0], np.cumsum(n)[:-1]]).astype(np.int32) if n else np.zeros(0, np.int32)
    return off, int(sum(n))


# ------------------------------------------------------------------ CPU reference
def recurrence_ref(q, k, v, g, beta, segs, scale, delta, init_state=None, init_idx=None):
    """Token-by-token reference; returns (o [rows, H*d], final [n_seg, H, d, d])."""
    rows, Hd = q.shape
    H = g.shape[1]
    d = Hd // H
    o = torch.zeros(rows, H, d, dtype=q.dtype)
    finals = []
    qh, kh, vh = q.view(rows, H, d), k.view(rows, H, d), v.view(rows, H, d)
    for s, (t0, T) in enumerate(segs):
        if init_state is not None and init_idx is not None and int(init_idx[s]) >= 0:
            S = init_state[int(init_idx[s])].clone()
        else:
            S = torch.zeros(H, d, d, dtype=q.dtype)
        for t in range(int(t0), int(t0) + int(T)):
            a = torch.exp(g[t]).view(H, 1, 1)
            kt = kh[t]
            if delta:
                u = torch.einsum("hji,hi->hj", S, kt)
                dd = beta[t].view(H, 1) * (vh[t] - a.view(H, 1) * u)
            else:
                dd = vh[t]
            S = a * S + dd.unsqueeze(-1) * kt.unsqueeze(1)
            o[t] = scale * torch.einsum("hji,hi->hj", S, qh[t])
        finals.append(S)
    return o.view(rows, Hd), (torch.stack(finals) if finals else torch.zeros(0, H, d, d, dtype=q.dtype))


def recurrence_chunked(q, k, v, g, beta, segs, scale, delta, init_state=None, init_idx=None, chunk: int = 64):
    """The same recurrence in chunks of `chunk` tokens (the chunked gated delta rule of
    Yang et al., "Gated Delta Networks", 2024, via its UT transform; GLA without the delta
    term), differentiable with plain tensor ops.

    Per head, a chunk with state S0 [d_v, d_k], cumulative log decay b_t (gamma_t = exp b_t)
    and R[t, s] = exp(b_t - b_s):
        A = strictly-lower(beta_t (k_t . k_s) R[t, s]),  (I + A) U = beta V,  (I + A) W = beta gamma K
        V' = U - W S0^T                                  (delta rule; GLA: V' = V)
        O  = scale ((gamma Q) S0^T + ((Q K^T) * lower-incl(R)) V')
        S  = gamma_L S0 + (V' * R[L, :])^T K
    Returns (o [rows, H*d], final [n_seg, H, d, d]) like recurrence_ref."""
    rows, Hd = q.shape
    H = g.shape[1]
    d = Hd // H
    dt = q.dtype if q.dtype == torch.float64 else torch.float32
    qh, kh, vh = (t.view(rows, H, d).to(dt) for t in (q, k, v))
    gh, bh = g.to(dt), beta.to(dt)
    out = torch.zeros(rows, H, d, dtype=dt, device=q.device)
    finals = []
    for s_idx, (t0, T) in enumerate(segs):
        t0, T = int(t0), int(T)
        if init_state is not None and init_idx is not None and int(init_idx[s_idx]) >= 0:
            S = init_state[int(init_idx[s_idx])].to(dt)
        else:
            S = torch.zeros(H, d, d, dtype=dt, device=q.device)
        for c0 in range(t0, t0 + T, chunk):
            c1 = min(t0 + T, c0 + chunk)
            L = c1 - c0
            Q, K, V = (x[c0:c1].transpose(0, 1) for x in (qh, kh, vh))   # [H, L, d]
            b = gh[c0:c1].transpose(0, 1).cumsum(-1)                     # [H, L]
            incl = torch.ones(L, L, dtype=torch.bool, device=q.device).tril()
            # the exponent is masked before exp: above the diagonal b_t - b_s > 0 can overflow,
            # and an inf there would turn the masked entries' gradients into NaN
            diff = (b[:, :, None] - b[:, None, :]).masked_fill(~incl, float("-inf"))
            R = torch.exp(diff)                                         # [H, L, L], 0 above the diagonal
            gam = torch.exp(b)                                           # [H, L]
            if delta:
                be = bh[c0:c1].transpose(0, 1)                           # [H, L]
                A = (be[:, :, None] * (K @ K.transpose(1, 2)) * R).tril(-1)
                I = torch.eye(L, dtype=dt, device=q.device).expand(H, L, L)
                U = torch.linalg.solve_triangular(I + A, be[:, :, None] * V, upper=False, unitriangular=True)
                W = torch.linalg.solve_triangular(I + A, (be * gam)[:, :, None] * K, upper=False,
                                                  unitriangular=True)
                Vp = U - W @ S.transpose(1, 2)
            else:
                Vp = V
            O = (gam[:, :, None] * Q) @ S.transpose(1, 2) + ((Q @ K.transpose(1, 2)) * R) @ Vp
            out[c0:c1] = (scale * O).transpose(0, 1)
            S = gam[:, -1, None, None] * S + (Vp * R[:, -1, :, None]).transpose(1, 2) @ K
        finals.append(S)
    fin = torch.stack(finals) if finals else torch.zeros(0, H, d, d, dtype=dt, device=q.device)
    return out.view(rows, Hd).to(q.dtype), fin


def conv_ref(x, w, bias, segs, ctx=None, ctx_idx=None, silu=True):
    rows, C = x.shape
    W = w.shape[1]
    y = torch.zeros_like(x)
    for s, (t0, T) in enumerate(segs):
        t0, T = int(t0), int(T)
        if ctx is not None and ctx_idx is not None and int(ctx_idx[s]) >= 0:
            pre = ctx[int(ctx_idx[s])].to(x.dtype)
        else:
            pre = torch.zeros(W - 1, C, dtype=x.dtype)
        xs = torch.cat([pre, x[t0:t0 + T]])
        acc = sum(xs[w_: w_ + T] * w[:, w_].to(x.dtype) for w_ in range(W))
        if bias is not None:
            acc = acc + bias.to(x.dtype)
        y[t0:t0 + T] = acc * torch.sigmoid(acc) if silu else acc
    return y


# ------------------------------------------------------------------ autograd
class _Recurrence(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, g, beta, init_state, segs, scale, delta, init_idx):
        ctx.segs, ctx.scale, ctx.delta, ctx.init_idx = segs, scale, delta, init_idx
        if not q.is_cuda or _chunked_on_gpu():
            o, fin = recurrence_chunked(q, k, v, g, beta, segs, scale, delta, init_state, init_idx)
            ctx.save_for_backward(q, k, v, g, beta, init_state)
            ctx.cpu = True
            return o, fin.to(torch.float64 if q.dtype == torch.float64 else torch.float32)
        ctx.cpu = False
        dev = q.device
        seg_t = _seg_tensor(segs, dev)
        off, n_ck = _ckpt_offsets(segs, ext().recur_chunk())
        off_t = torch.from_numpy(off).to(dev)
        idx_t = torch.as_tensor(np.asarray(init_idx, np.int32), device=dev) if init_state is not None else None
        o, fin, ck = ext().recur_fwd(q, k, v, g.contiguous(), beta.contiguous() if delta else None, seg_t, g.shape[1],
                                     scale, delta, init_state, idx_t, off_t, n_ck)
        ctx.save_for_backward(q, k, v, g, beta, init_state, ck)
        ctx.aux = (seg_t, off_t, idx_t)
        return o, fin

    @staticmethod
    def backward(ctx, do, dfin):
        if ctx.cpu:
            q, k, v, g, beta, init_state = ctx.saved_tensors
            with torch.enable_grad():
                ins = [t.detach().requires_grad_(True) if t is not None else None
                       for t in (q, k, v, g, beta, init_state)]
                o, fin = recurrence_chunked(*ins[:5], ctx.segs, ctx.scale, ctx.delta, ins[5], ctx.init_idx)
                outs, grads = [o], [do]
                if dfin is not None:
                    outs.append(fin)
                    grads.append(dfin)
                req = [t for t in ins if t is not None and t.requires_grad]
                got = torch.autograd.grad(outs, req, grads, allow_unused=True)
            it = iter(got)
            res = [next(it) if t is not None else None for t in ins]
            return (*res, None, None, None, None)
        q, k, v, g, beta, init_state, ck = ctx.saved_tensors
        seg_t, off_t, idx_t = ctx.aux
        dq, dk, dv, dg, dbeta, dinit = ext().recur_bwd(q, k, v, g.contiguous(),
                                                       beta.contiguous() if ctx.delta else None, seg_t, g.shape[1],
                                                       ctx.scale, ctx.delta, init_state, idx_t, off_t, ck,
                                                       do.contiguous(), dfin.contiguous() if dfin is not None else None)
        d_init_state = None
        if init_state is not None:
            d_init_state = torch.zeros_like(init_state)
            ii = torch.as_tensor(np.asarray(ctx.init_idx, np.int64), device=q.device)
            ok = ii >= 0
            d_init_state.index_add_(0, ii[ok], dinit[ok])
        return dq, dk, dv, dg, (dbeta if ctx.delta else None), d_init_state, None, None, None, None


def _chunked_on_gpu() -> bool:
    """OCTO_RECURRENCE_CHUNKED=1: CUDA tensors take the chunked tensor-op form (batched GEMMs
    and triangular solves) instead of the token-serial kernels."""
    import os

    return os.environ.get("OCTO_RECURRENCE_CHUNKED", "0") == "1"


def recurrence(q, k, v, g, beta, segs, scale: float, delta: bool, init_state=None, init_idx=None):
    """(o, final) of the gated delta rule (delta=True) or simple GLA (delta=False)."""
    if beta is None:
        beta = g.new_zeros(g.shape)
    return _Recurrence.apply(q, k, v, g, beta, init_state, [tuple(map(int, s)) for s in segs], float(scale),
                             bool(delta), None if init_idx is None else [int(i) for i in init_idx])


class _Conv(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, bias, cx, segs, ctx_idx, silu):
        ctx.segs, ctx.ctx_idx, ctx.silu = segs, ctx_idx, silu
        ctx.save_for_backward(x, w, bias, cx)
        if not x.is_cuda:
            return conv_ref(x, w, bias, segs, cx, ctx_idx, silu)
        cu = torch.as_tensor(np.r_[0, np.cumsum([int(l) for _, l in segs])].astype(np.int32), device=x.device)
        ctx.cu = cu
        ci = torch.as_tensor(np.asarray(ctx_idx, np.int32), device=x.device) if cx is not None else None
        ctx.ci = ci
        return ext().conv_fwd(x.contiguous(), w.contiguous(), bias, cu, cx, ci, silu)

    @staticmethod
    def backward(ctx, dy):
        x, w, bias, cx = ctx.saved_tensors
        if not x.is_cuda:
            with torch.enable_grad():
                ins = [t.detach().requires_grad_(True) if t is not None else None for t in (x, w, bias, cx)]
                y = conv_ref(ins[0], ins[1], ins[2], ctx.segs, ins[3], ctx.ctx_idx, ctx.silu)
                req = [t for t in ins if t is not None]
                got = torch.autograd.grad(y, req, dy, allow_unused=True)
            it = iter(got)
            res = [next(it) if t is not None else None for t in ins]
            return (*res, None, None, None)
        dx, dw, db, dctx = ext().conv_bwd(x.contiguous(), w.contiguous(), bias, ctx.cu, cx, ctx.ci, ctx.silu,
                                          dy.contiguous())
        d_cx = None
        if cx is not None:
            d_cx = torch.zeros_like(cx)
            ii = torch.as_tensor(np.asarray(ctx.ctx_idx, np.int64), device=x.device)
            ok = ii >= 0
            d_cx.index_add_(0, ii[ok], dctx[ok])
        return dx, dw, (db if bias is not None else None), d_cx, None, None, None


def causal_conv(x, w, bias, segs, ctx=None, ctx_idx=None, silu: bool = True):
    """Causal depthwise conv over contiguous segments (segs: [(start, len)] covering x in order)."""
    segs = [tuple(map(int, s)) for s in segs]
    return _Conv.apply(x, w, bias, ctx, segs, None if ctx_idx is None else [int(i) for i in ctx_idx], bool(silu))
