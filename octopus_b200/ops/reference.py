"""Plain-PyTorch reference implementations of every kernel (CPU path and test oracle).

Each function computes in fp32 (or the input dtype when it is fp64) and mirrors the
semantics of the corresponding sm_100a kernel exactly:

* ``linear``            y = x W^T (+ b) (+ residual)
* ``rmsnorm``           y = x * rsqrt(mean(x^2) + eps) * (w | 1 + w)
* ``rope``              neox rotate-half rotary embedding at integer positions
* ``swiglu``            silu(gate) * up for gu = [gate | up]
* ``gather_attention``  per-sequence softmax attention over a gathered key list with
                        bottom-right causal alignment (query i of n_q sees key j of n_k
                        iff j <= n_k - n_q + i), GQA by head grouping
* ``logprob_head``      (log p(label), entropy) of softmax(alpha * h W^T)
"""
from __future__ import annotations

import math

import torch


def _f(x: torch.Tensor) -> torch.Tensor:
    return x if x.dtype == torch.float64 else x.float()


def linear(x, w, bias=None, residual=None):
    y = _f(x) @ _f(w).t()
    if bias is not None:
        y = y + _f(bias)
    if residual is not None:
        y = y + _f(residual)
    return y


def rmsnorm(x, w, eps: float, plus_one: bool = False):
    xf = _f(x)
    r = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    wf = _f(w)
    return xf * r * ((1.0 + wf) if plus_one else wf)


def rope_cos_sin(pos: torch.Tensor, dim: int, theta: float, dtype=torch.float32):
    inv = theta ** (-torch.arange(0, dim, 2, dtype=torch.float64, device=pos.device) / dim)
    ang = pos.to(torch.float64)[:, None] * inv[None, :]
    return ang.cos().to(dtype), ang.sin().to(dtype)


def rope(x: torch.Tensor, pos: torch.Tensor, theta: float, inverse: bool = False):
    """x: [T, H, D]; rotate-half convention."""
    D = x.shape[-1]
    cos, sin = rope_cos_sin(pos, D, theta, dtype=_f(x).dtype)
    if inverse:
        sin = -sin
    xf = _f(x)
    a, b = xf[..., : D // 2], xf[..., D // 2:]
    c, s = cos[:, None, :], sin[:, None, :]
    return torch.cat([a * c - b * s, b * c + a * s], dim=-1)


def swiglu(gu: torch.Tensor):
    g, u = _f(gu).chunk(2, dim=-1)
    return torch.nn.functional.silu(g) * u


def gather_attention(q, k, v, cu_q, cu_k, key_idx, scale: float, causal: bool = True):
    """q: [Tq, Hq, D], k/v: [rows, Hkv, D] -> o [Tq, Hq, D], lse [Hq, Tq] (fp32/fp64)."""
    Tq, Hq, D = q.shape
    Hkv = k.shape[1]
    G = Hq // Hkv
    dt = torch.float64 if q.dtype == torch.float64 else torch.float32
    o = torch.zeros(Tq, Hq, D, dtype=dt, device=q.device)
    lse = torch.full((Hq, Tq), -math.inf, dtype=dt, device=q.device)
    cu_q = [int(x) for x in cu_q]
    cu_k = [int(x) for x in cu_k]
    for s in range(len(cu_q) - 1):
        qa, qb = cu_q[s], cu_q[s + 1]
        ka, kb = cu_k[s], cu_k[s + 1]
        nq, nk = qb - qa, kb - ka
        if nq == 0:
            continue
        idx = key_idx[ka:kb].long()
        qs = q[qa:qb].to(dt)
        ks = k[idx].to(dt).repeat_interleave(G, dim=1)
        vs = v[idx].to(dt).repeat_interleave(G, dim=1)
        sc = torch.einsum("qhd,khd->hqk", qs, ks) * scale
        if causal:
            i = torch.arange(nq, device=q.device)[:, None]
            j = torch.arange(nk, device=q.device)[None, :]
            sc = sc.masked_fill(j > (nk - nq + i), -math.inf)
        l = torch.logsumexp(sc, dim=-1)
        p = torch.exp(sc - l[..., None])
        p = torch.nan_to_num(p, nan=0.0)
        o[qa:qb] = torch.einsum("hqk,khd->qhd", p, vs)
        lse[:, qa:qb] = l
    return o, lse


def logprob_head(h, W, labels, alpha: float = 1.0, vocab_limit: int | None = None, vocab_chunk: int = 0):
    """Returns (logp [M], entropy [M], lse [M]); rows with label < 0 get logp 0.

    vocab_chunk > 0 computes the normaliser chunk by chunk over the vocabulary with an
    online (max, sum exp, sum exp*z) merge, as the fused kernel does per vocab tile.
    """
    if vocab_chunk:
        return _logprob_head_chunked(h, W, labels, alpha, vocab_limit, vocab_chunk)
    z = (_f(h) @ _f(W).t()) * alpha
    if vocab_limit is not None and vocab_limit < z.shape[1]:
        z = z[:, :vocab_limit]
    lse = torch.logsumexp(z, dim=-1)
    lp = z - lse[:, None]
    p = lp.exp()
    ent = -(p * lp).sum(-1)
    lab = labels.long()
    picked = torch.where(lab >= 0, lp.gather(1, lab.clamp(min=0)[:, None])[:, 0], torch.zeros_like(lse))
    return picked, ent, lse


def _logprob_head_chunked(h, W, labels, alpha, vocab_limit, chunk):
    hf = _f(h)
    V = vocab_limit or W.shape[0]
    M = hf.shape[0]
    m = torch.full((M,), -math.inf, dtype=hf.dtype)
    s = torch.zeros(M, dtype=hf.dtype)
    t = torch.zeros(M, dtype=hf.dtype)
    zl = torch.zeros(M, dtype=hf.dtype)
    lab = labels.long()
    for a in range(0, V, chunk):
        b = min(V, a + chunk)
        z = (hf @ _f(W[a:b]).t()) * alpha
        cm = z.max(-1).values
        nm = torch.maximum(m, cm)
        sc = torch.exp(m - nm)
        e = torch.exp(z - nm[:, None])
        s = s * sc + e.sum(-1)
        t = t * sc + (e * z).sum(-1)
        m = nm
        inside = (lab >= a) & (lab < b)
        zl = torch.where(inside, z.gather(1, (lab - a).clamp(0, b - a - 1)[:, None])[:, 0], zl)
    lse = m + torch.log(s)
    logp = torch.where(lab >= 0, zl - lse, torch.zeros_like(lse))
    ent = lse - t / s
    return logp, ent, lse
