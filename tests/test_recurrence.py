"""Linear recurrences and causal conv (hybrid models): CPU semantics and, on a GPU, the
sm_100a kernels against the token-by-token fp32 references (outputs, final states and
gradients, with initial states and several segments)."""
import numpy as np
import pytest
import torch

from octopus_b200.ops.recurrence import causal_conv, conv_ref, recurrence, recurrence_ref


def _inputs(rows, H, d, dtype, seed=0, device="cpu"):
    g = torch.Generator().manual_seed(seed)
    q = torch.nn.functional.normalize(torch.randn(rows, H, d, generator=g, dtype=torch.float64), dim=-1)
    k = torch.nn.functional.normalize(torch.randn(rows, H, d, generator=g, dtype=torch.float64), dim=-1)
    v = torch.randn(rows, H, d, generator=g, dtype=torch.float64)
    gg = -torch.rand(rows, H, generator=g, dtype=torch.float64) * 0.3
    beta = torch.sigmoid(torch.randn(rows, H, generator=g, dtype=torch.float64))
    f = lambda t: t.to(dtype).to(device)  # noqa: E731
    return f(q.reshape(rows, -1)), f(k.reshape(rows, -1)), f(v.reshape(rows, -1)), gg.float().to(device), \
        beta.float().to(device)


@pytest.mark.parametrize("delta", [True, False])
def test_tree_states_equal_concatenated_sequence(delta):
    """A segment started from its parent's final state continues the parent exactly."""
    q, k, v, g, b = _inputs(30, 2, 8, torch.float64)
    g, b = g.double(), b.double()
    o_full, fin_full = recurrence(q, k, v, g, b, [(0, 30)], 0.5, delta)
    o1, f1 = recurrence(q[:12], k[:12], v[:12], g[:12], b[:12], [(0, 12)], 0.5, delta)
    o2, f2 = recurrence(q[12:], k[12:], v[12:], g[12:], b[12:], [(0, 18)], 0.5, delta, init_state=f1,
                        init_idx=[0])
    assert torch.allclose(torch.cat([o1, o2]), o_full) and torch.allclose(f2, fin_full)


def test_recurrence_gradients_cpu():
    q, k, v, g, b = _inputs(9, 1, 4, torch.float64)
    g, b = g.double(), b.double()
    init = torch.randn(1, 1, 4, 4, dtype=torch.float64)
    ins = [t.requires_grad_(True) for t in (q, k, v, g, b, init)]

    def f(q, k, v, g, b, init):
        o, fin = recurrence(q, k, v, g, b, [(0, 5), (5, 4)], 0.7, True, init_state=init, init_idx=[0, -1])
        return o.sum() + (fin ** 2).sum()

    assert torch.autograd.gradcheck(f, ins, eps=1e-6, atol=1e-5)


def test_conv_context_equals_concatenation():
    x = torch.randn(20, 6, dtype=torch.float64)
    w = torch.randn(6, 4, dtype=torch.float64)
    b = torch.randn(6, dtype=torch.float64)
    full = causal_conv(x, w, b, [(0, 20)])
    ctx = x[5:8].unsqueeze(0)  # the 3 rows before the second segment
    part = causal_conv(x[8:], w, b, [(0, 12)], ctx=ctx, ctx_idx=[0])
    assert torch.allclose(part, full[8:])


@pytest.mark.gpu
@pytest.mark.parametrize("delta,d", [(True, 128), (False, 128), (True, 64)])
def test_recurrence_cuda_matches_reference(delta, d):
    dev = torch.device("cuda", 0)
    H, rows = 2, 70
    segs = [(0, 33), (33, 37)]
    q, k, v, g, b = _inputs(rows, H, d, torch.bfloat16, seed=3, device=dev)
    init = (torch.randn(1, H, d, d, device=dev) * 0.1)
    ins = [t.detach().clone().requires_grad_(True) for t in (q, k, v, g, b, init)]
    o, fin = recurrence(*ins[:5], segs, d ** -0.5, delta, init_state=ins[5], init_idx=[0, -1])
    do = torch.randn_like(o)
    dfin = torch.randn_like(fin) * 0.1
    torch.autograd.backward([o, fin], [do, dfin])
    refs = [t.detach().float().cpu().requires_grad_(True) for t in (q, k, v, g, b, init)]
    o_r, fin_r = recurrence_ref(*refs[:5], segs, d ** -0.5, delta, refs[5], [0, -1])
    torch.autograd.backward([o_r, fin_r], [do.float().cpu(), dfin.cpu()])

    def rel(a, b_):
        a, b_ = a.float().cpu(), b_.float().cpu()
        return float((a - b_).abs().max() / b_.abs().max().clamp_min(1e-6))

    assert rel(o, o_r) < 2e-2 and rel(fin, fin_r) < 1e-2
    names = ["q", "k", "v", "g", "beta", "init"]
    for n, a, r in zip(names, ins, refs):
        if n == "beta" and not delta:
            continue
        assert rel(a.grad, r.grad) < 3e-2, n


@pytest.mark.gpu
def test_conv_cuda_matches_reference():
    dev = torch.device("cuda", 0)
    rows, C, W = 50, 256, 4
    x = torch.randn(rows, C, device=dev).bfloat16().requires_grad_(True)
    w = torch.randn(C, W, device=dev).requires_grad_(True)
    b = torch.randn(C, device=dev).requires_grad_(True)
    ctx = torch.randn(2, W - 1, C, device=dev).requires_grad_(True)
    segs = [(0, 20), (20, 30)]
    y = causal_conv(x, w, b, segs, ctx=ctx, ctx_idx=[1, -1])
    dy = torch.randn_like(y)
    y.backward(dy)
    xr, wr, br, cr = (t.detach().float().cpu().requires_grad_(True) for t in (x, w, b, ctx))
    yr = conv_ref(xr, wr, br, segs, cr, [1, -1])
    yr.backward(dy.float().cpu())
    assert float((y.float().cpu() - yr).abs().max()) < 5e-2
    for a, r in ((x, xr), (w, wr), (b, br), (ctx, cr)):
        assert float((a.grad.float().cpu() - r.grad).abs().max() / r.grad.abs().max()) < 2e-2


def _rand(rows, H, d, dtype, seed, decay=0.5):
    gen = torch.Generator().manual_seed(seed)
    nq = lambda: torch.nn.functional.normalize(torch.randn(rows, H, d, generator=gen, dtype=dtype), dim=-1)  # noqa
    q, k = nq().reshape(rows, H * d), nq().reshape(rows, H * d)
    v = torch.randn(rows, H * d, generator=gen, dtype=dtype)
    g = -torch.rand(rows, H, generator=gen, dtype=dtype) * decay
    beta = torch.rand(rows, H, generator=gen, dtype=dtype)
    init = torch.randn(2, H, d, d, generator=gen, dtype=dtype) * 0.3
    return q, k, v, g, beta, init


@pytest.mark.parametrize("delta", [True, False])
@pytest.mark.parametrize("chunk", [1, 7, 16, 64])
def test_chunked_equals_token_serial(delta, chunk):
    """The chunked (UT-transform) form equals the token-by-token recurrence: outputs, final
    states and every input gradient (initial states included), over ragged segments."""
    from octopus_b200.ops.recurrence import recurrence_chunked

    rows, H, d = 150, 2, 8
    segs = [(0, 1), (1, 63), (64, 65), (129, 21)]
    idx = [1, -1, 0, 1]
    base = _rand(rows, H, d, torch.float64, 0)
    res = []
    for fn in (recurrence_ref, lambda *a: recurrence_chunked(*a, chunk=chunk)):
        ins = [t.clone().requires_grad_(True) for t in base]
        o, fin = fn(*ins[:5], segs, d ** -0.5, delta, ins[5], idx)
        gen = torch.Generator().manual_seed(1)
        (o * torch.randn(o.shape, generator=gen, dtype=o.dtype)).sum().backward(retain_graph=True)
        (fin * 0.37).sum().backward()
        res.append((o.detach(), fin.detach(), [t.grad for t in ins]))
    (o1, f1, g1), (o2, f2, g2) = res
    assert torch.allclose(o1, o2, atol=1e-12) and torch.allclose(f1, f2, atol=1e-12)
    for a, b in zip(g1, g2):
        if a is None or b is None:
            assert a is None or float(a.abs().max()) == 0.0
            continue
        assert torch.allclose(a, b, atol=1e-10)


def test_chunked_fp32_strong_decay_gradients_finite():
    """Strong decays (exponents past fp32 range above the diagonal) keep finite gradients."""
    from octopus_b200.ops.recurrence import recurrence_chunked

    ins = [t.float().requires_grad_(True) for t in _rand(80, 2, 8, torch.float64, 3, decay=40.0)]
    o, fin = recurrence_chunked(*ins[:5], [(0, 80)], 8 ** -0.5, True, ins[5], [0], chunk=64)
    (o.sum() + fin.sum()).backward()
    assert all(torch.isfinite(t.grad).all() for t in ins)


@pytest.mark.gpu
def test_chunked_tensor_ops_on_gpu_match_kernel(monkeypatch):
    """OCTO_RECURRENCE_CHUNKED=1 on CUDA (tensor ops) against the token-serial sm_100a kernel."""
    dev = torch.device("cuda", 0)
    q, k, v, g, b = _inputs(70, 2, 128, torch.bfloat16, seed=5, device=dev)
    init = torch.randn(1, 2, 128, 128, device=dev) * 0.1
    segs = [(0, 33), (33, 37)]
    o1, f1 = recurrence(q, k, v, g, b, segs, 128 ** -0.5, True, init_state=init, init_idx=[0, -1])
    monkeypatch.setenv("OCTO_RECURRENCE_CHUNKED", "1")
    o2, f2 = recurrence(q, k, v, g, b, segs, 128 ** -0.5, True, init_state=init, init_idx=[0, -1])
    torch.cuda.synchronize()
    rel = lambda a, c: float((a.float() - c.float()).norm() / (c.float().norm() + 1e-12))  # noqa: E731
    assert rel(o2, o1) < 2e-2 and rel(f2, f1) < 2e-2
