"""GPU numerics of every sm_100a kernel against plain-PyTorch fp32 references."""
import math

import numpy as np
import pytest
import torch

from octopus_b200 import ops
from octopus_b200.ops import reference as ref

pytestmark = pytest.mark.gpu
dev = "cuda"


def rel_err(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / (b.norm() + 1e-12))


@pytest.fixture(autouse=True)
def _status():
    yield
    ops.check_status(0)


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 1024), (1000, 1536, 1536), (40, 200, 96),
                                   (4096, 4608, 3584)])
@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, False), (True, True)])
def test_gemm(M, N, K, a_mn, b_mn):
    torch.manual_seed(0)
    A = torch.randn(M, K, device=dev).bfloat16()
    B = torch.randn(N, K, device=dev).bfloat16()
    a = A.t().contiguous() if a_mn else A
    b = B.t().contiguous() if b_mn else B
    C = ops.gemm(a, b, a_mn=a_mn, b_mn=b_mn)
    R = A.float() @ B.float().t()
    assert rel_err(C, R) < 1e-2


@pytest.mark.parametrize("bn", [64, 128, 256])
def test_gemm_tiles_and_epilogues(bn):
    torch.manual_seed(1)
    M, N, K = 520, 776, 512
    A = torch.randn(M, K, device=dev).bfloat16()
    B = torch.randn(N, K, device=dev).bfloat16()
    bias = torch.randn(N, device=dev).bfloat16()
    res = torch.randn(M, N, device=dev).bfloat16()
    C = ops.gemm(A, B, bias=bias, residual=res, alpha=0.5, bn=bn)
    R = 0.5 * (A.float() @ B.float().t()) + bias.float() + res.float()
    assert rel_err(C, R) < 1e-2
    acc = torch.randn(M, N, device=dev)
    base = acc.clone()
    ops.gemm(A, B, out=acc, accumulate=True, bn=bn)
    assert rel_err(acc, base + A.float() @ B.float().t()) < 1e-2


def test_linear_autograd():
    torch.manual_seed(2)
    x = torch.randn(384, 512, device=dev).bfloat16().requires_grad_(True)
    w = torch.randn(768, 512, device=dev).bfloat16() * 0.05
    w.main_grad = torch.zeros(768, 512, device=dev)
    b = torch.randn(768, device=dev).bfloat16()
    b.main_grad = torch.zeros(768, device=dev)
    y = ops.linear(x, w, b)
    g = torch.randn_like(y)
    y.backward(g)
    xr = x.detach().float().requires_grad_(True)
    wr = w.float().requires_grad_(True)
    yr = xr @ wr.t() + b.float()
    yr.backward(g.float())
    assert rel_err(y, yr) < 1e-2
    assert rel_err(x.grad, xr.grad) < 1e-2
    assert rel_err(w.main_grad, wr.grad) < 1e-2
    assert rel_err(b.main_grad, g.float().sum(0)) < 1e-3


def test_rmsnorm_fwd_bwd():
    torch.manual_seed(3)
    for plus_one in (False, True):
        x = torch.randn(333, 1536, device=dev).bfloat16().requires_grad_(True)
        w = (torch.rand(1536, device=dev) + 0.5).bfloat16()
        w.main_grad = torch.zeros(1536, device=dev)
        y = ops.rmsnorm(x, w, 1e-6, plus_one)
        g = torch.randn_like(y)
        y.backward(g)
        xr = x.detach().float().requires_grad_(True)
        wr = w.float().requires_grad_(True)
        yr = ref.rmsnorm(xr, wr, 1e-6, plus_one)
        yr.backward(g.float())
        assert rel_err(y, yr) < 1e-2
        assert rel_err(x.grad, xr.grad) < 2e-2
        assert rel_err(w.main_grad, wr.grad) < 2e-2


def test_rope_roundtrip():
    torch.manual_seed(4)
    T, Hq, Hkv, D = 77, 4, 2, 128
    qkv = torch.randn(T, (Hq + 2 * Hkv) * D, device=dev).bfloat16()
    pos = torch.randint(0, 30000, (T,), device=dev, dtype=torch.int32)
    x = qkv.clone()
    ops.ext().rope(x, pos, Hq, Hkv, D, 1e6, False)
    r = ref.rope(qkv[:, : (Hq + Hkv) * D].reshape(T, Hq + Hkv, D).cpu(), pos.cpu(), 1e6)
    assert rel_err(x[:, : (Hq + Hkv) * D].reshape(T, Hq + Hkv, D).cpu(), r) < 1e-2
    assert torch.equal(x[:, (Hq + Hkv) * D:], qkv[:, (Hq + Hkv) * D:])
    ops.ext().rope(x, pos, Hq, Hkv, D, 1e6, True)
    assert rel_err(x, qkv) < 2e-2


def test_swiglu():
    torch.manual_seed(5)
    gu = torch.randn(100, 2 * 688, device=dev).bfloat16().requires_grad_(True)
    y = ops.swiglu(gu)
    g = torch.randn_like(y)
    y.backward(g)
    gr = gu.detach().float().requires_grad_(True)
    yr = ref.swiglu(gr)
    yr.backward(g.float())
    assert rel_err(y, yr) < 1e-2
    assert rel_err(gu.grad, gr.grad) < 2e-2


def _tree_plan(rng, n_nodes=12, H=64):
    """Random tree: each node = parent path keys + own rows (own last), rows contiguous."""
    lens = rng.integers(1, 300, size=n_nodes)
    parent = [-1] + [int(rng.integers(0, i)) for i in range(1, n_nodes)]
    starts = np.concatenate([[0], np.cumsum(lens)[:-1]])
    keys, cu_k, cu_q = [], [0], [0]
    for i in range(n_nodes):
        path = []
        p = parent[i]
        chain = []
        while p >= 0:
            chain.append(p)
            p = parent[p]
        for a in reversed(chain):
            path.extend(range(starts[a], starts[a] + lens[a]))
        path.extend(range(starts[i], starts[i] + lens[i]))
        keys.extend(path)
        cu_k.append(len(keys))
        cu_q.append(cu_q[-1] + lens[i])
    return int(lens.sum()), cu_q, cu_k, np.asarray(keys, dtype=np.int32)


@pytest.mark.parametrize("D,Hq,Hkv", [(128, 28, 4), (64, 4, 4), (128, 12, 2)])
def test_tree_attention_fwd_bwd(D, Hq, Hkv):
    rng = np.random.default_rng(6)
    torch.manual_seed(6)
    T, cu_q, cu_k, keys = _tree_plan(rng)
    plan = ops.AttnPlan.build(cu_q, cu_k, keys, dev)
    qkv = (torch.randn(T, (Hq + 2 * Hkv) * D, device=dev) * 0.5).bfloat16().requires_grad_(True)
    o = ops.attention(qkv, plan, Hq, Hkv, D)
    g = torch.randn_like(o)
    o.backward(g)
    x = qkv.detach().float().cpu().requires_grad_(True)
    q = x[:, : Hq * D].reshape(T, Hq, D)
    k = x[:, Hq * D: (Hq + Hkv) * D].reshape(T, Hkv, D)
    v = x[:, (Hq + Hkv) * D:].reshape(T, Hkv, D)
    orf, _ = ref.gather_attention(q, k, v, cu_q, cu_k, torch.from_numpy(keys), D ** -0.5)
    orf = orf.reshape(T, Hq * D)
    orf.backward(g.float().cpu())
    assert rel_err(o.cpu(), orf) < 2e-2
    assert rel_err(qkv.grad.cpu(), x.grad) < 3e-2


def test_decode_attention():
    torch.manual_seed(7)
    B, Hq, Hkv, D = 37, 28, 4, 128
    slots = 6000
    kc = torch.randn(slots, Hkv * D, device=dev).bfloat16()
    vc = torch.randn(slots, Hkv * D, device=dev).bfloat16()
    lens = torch.randint(1, 1500, (B,))
    ip = torch.zeros(B + 1, dtype=torch.int32)
    ip[1:] = torch.cumsum(lens, 0)
    idx = torch.randint(0, slots, (int(ip[-1]),), dtype=torch.int32)
    q = torch.randn(B, Hq * D, device=dev).bfloat16()
    for splits in (1, 4):
        da = ops.DecodeAttention(Hq, Hkv, D, B, splits, dev)
        o = da(q, kc, vc, ip.to(dev), idx.to(dev))
        r = ops.decode.decode_attention_ref(q.cpu().float(), kc.cpu().float(), vc.cpu().float(), ip, idx, Hq, Hkv,
                                            D, D ** -0.5)
        assert rel_err(o.cpu(), r) < 2e-2


def test_logprob_head_fwd_bwd():
    torch.manual_seed(8)
    M, H, V = 1000, 512, 5000
    h = (torch.randn(M, H, device=dev) * 0.5).bfloat16().requires_grad_(True)
    W = (torch.randn(V + 120, H, device=dev) * 0.05).bfloat16()
    W.main_grad = torch.zeros(W.shape, device=dev)
    labels = torch.randint(0, V, (M,), device=dev)
    labels[::7] = -1
    lp, ent = ops.logprob_head(h, W, labels, 0.8, V)
    glp, gent = torch.randn(M, device=dev), torch.randn(M, device=dev) * 0.1
    (lp * glp + ent * gent).sum().backward()
    hr = h.detach().float().requires_grad_(True)
    Wr = W.float().requires_grad_(True)
    lpr, entr, _ = ref.logprob_head(hr, Wr, labels, 0.8, V)
    (lpr * glp + entr * gent).sum().backward()
    assert rel_err(lp, lpr) < 1e-2
    assert rel_err(ent, entr) < 1e-2
    assert rel_err(h.grad, hr.grad) < 3e-2
    assert rel_err(W.main_grad, Wr.grad) < 3e-2


def test_empty_rows_head_and_gemm():
    """Zero-row operands (a rank's empty micro-batch) return empty results and zero gradients
    without building a tensor map or launching a kernel."""
    H, V = 512, 1024
    h = torch.zeros(0, H, device=dev, dtype=torch.bfloat16, requires_grad=True)
    W = (torch.randn(V, H, device=dev) * 0.05).bfloat16().requires_grad_(True)
    lp, ent = ops.logprob_head(h, W, torch.zeros(0, dtype=torch.int64, device=dev), 1.0, V)
    assert lp.shape == (0,) and ent.shape == (0,)
    (lp.sum() + ent.sum()).backward()
    assert h.grad.shape == (0, H) and float(W.grad.float().abs().sum()) == 0.0
    y = ops.gemm(torch.zeros(0, H, device=dev, dtype=torch.bfloat16), W.detach())
    assert y.shape == (0, V)
    torch.cuda.synchronize()
    ops.check_status(0)


@pytest.mark.parametrize("M,F,K", [(8, 512, 256), (40, 1024, 512), (200, 1024, 512), (256, 18944, 3584),
                                   (1000, 1536, 768)])
def test_gemm_swiglu_matches_gemm_then_swiglu(M, F, K):
    """The gate / up GEMM with SwiGLU in its epilogue (paired 128-row gate and up tiles,
    decode-sized and large M) against the GEMM followed by the swiglu kernel, and against
    an fp32 reference."""
    torch.manual_seed(11)
    x = torch.randn(M, K, device=dev).bfloat16()
    W = (torch.randn(2 * F, K, device=dev) * K ** -0.5).bfloat16()
    fused = ops.gemm_swiglu(x, W)
    unfused = ops.swiglu(ops.gemm(x, W))
    torch.cuda.synchronize()
    ops.check_status(0)
    assert fused.shape == (M, F)
    assert (fused.float() - unfused.float()).abs().max().item() <= 1e-2 * unfused.float().abs().max().item()
    gu = x.float() @ W.float().t()
    g, u = gu[:, :F], gu[:, F:]
    want = g * torch.sigmoid(g) * u
    assert rel_err(fused, want) < 1e-2


@pytest.mark.parametrize("M,Hq,Hkv,D,bias", [(64, 4, 2, 64, True), (1000, 28, 4, 128, True), (264, 8, 8, 128, False)])
def test_linear_rope_matches_linear_then_rope(M, Hq, Hkv, D, bias):
    """The qkv projection with the rotary embedding in its epilogue: forward equals the GEMM
    followed by the rope kernel; gradients of x, W and the bias match the unfused ops."""
    torch.manual_seed(12)
    K, N = 256, (Hq + 2 * Hkv) * D
    x = torch.randn(M, K, device=dev).bfloat16().requires_grad_(True)
    W = (torch.randn(N, K, device=dev) * K ** -0.5).bfloat16().requires_grad_(True)
    b = (torch.randn(N, device=dev) * 0.1).bfloat16().requires_grad_(True) if bias else None
    pos = torch.randint(0, 4000, (M,), device=dev, dtype=torch.int32)
    y = ops.linear_rope(x, W, b, pos, Hq, Hkv, D, 1e6)
    x2 = x.detach().clone().requires_grad_(True)
    W2 = W.detach().clone().requires_grad_(True)
    b2 = b.detach().clone().requires_grad_(True) if bias else None
    y2 = ops.rope_(ops.linear(x2, W2, b2), pos, Hq, Hkv, D, 1e6)
    assert (y.float() - y2.float()).abs().max().item() <= 1e-2 * y2.float().abs().max().item()
    gy = torch.randn_like(y)
    y.backward(gy)
    y2.backward(gy)
    torch.cuda.synchronize()
    ops.check_status(0)
    assert rel_err(x.grad, x2.grad) < 1e-2
    assert rel_err(W.grad, W2.grad) < 1e-2
    if bias:
        assert rel_err(b.grad, b2.grad) < 1e-2


def test_sampling_distribution():
    torch.manual_seed(9)
    H, V = 64, 256
    W = torch.randn(V, H, device=dev).bfloat16() * 0.3
    h1 = torch.randn(1, H, device=dev).bfloat16()
    h = h1.repeat(8192, 1)
    streams = torch.arange(8192, device=dev, dtype=torch.int64)
    tok, lp = ops.sample(h, W, temperature=1.0, seed=1234, row_stream=streams)
    p = torch.softmax(h1.float() @ W.float().t(), -1)[0]
    emp = torch.bincount(tok, minlength=V).float() / tok.numel()
    assert float((emp - p).abs().sum()) < 0.15
    assert torch.allclose(lp, torch.log(p[tok]), atol=2e-2)
    tok2, _ = ops.sample(h, W, temperature=1.0, seed=1234, row_stream=streams)
    assert torch.equal(tok, tok2)


def test_adamw_matches_reference():
    torch.manual_seed(10)
    n = 10007
    p = torch.randn(n, device=dev)
    g = torch.randn(n, device=dev)
    m = torch.zeros(n, device=dev)
    v = torch.zeros(n, device=dev)
    p16 = torch.empty(n, device=dev, dtype=torch.bfloat16)
    sq = torch.zeros(1, device=dev)
    ops.sqnorm_(g, sq)
    assert abs(float(sq) - float((g * g).sum())) / float((g * g).sum()) < 1e-4
    pc, gc, mc, vc = p.cpu(), g.cpu(), m.cpu(), v.cpu()
    ops.adamw_(p, g, m, v, p16, lr=1e-3, weight_decay=0.1, step=1, sqnorm=sq, max_norm=1.0)
    ops.adamw_(pc, gc, mc, vc, None, lr=1e-3, weight_decay=0.1, step=1, sqnorm=sq.cpu(), max_norm=1.0)
    assert rel_err(p.cpu(), pc) < 1e-5
    assert rel_err(p16.float().cpu(), pc) < 1e-2


def test_embedding():
    torch.manual_seed(11)
    W = torch.randn(1000, 256, device=dev).bfloat16().requires_grad_(True)
    W.main_grad = torch.zeros(1000, 256, device=dev)
    ids = torch.randint(0, 1000, (300,), device=dev)
    y = ops.embed(ids, W)
    assert torch.equal(y, W.detach()[ids])
    g = torch.randn_like(y)
    y.backward(g)
    r = torch.zeros(1000, 256, device=dev).index_add_(0, ids, g.float())
    assert rel_err(W.main_grad, r) < 1e-3


def test_sampling_never_nan_over_many_rows():
    """Regression: the uniform variate must stay strictly inside (0, 1) (an exact 1.0 gave +inf noise)."""
    torch.manual_seed(12)
    H, V = 256, 152064
    W = (torch.randn(V, H, device=dev) * 0.05).bfloat16()
    h = torch.randn(512, H, device=dev).bfloat16()
    for seed in range(4):
        tok, lp = ops.sample(h, W, temperature=1.0, seed=seed,
                             row_stream=torch.arange(512, device=dev, dtype=torch.int64) + 1000 * seed)
        assert torch.isfinite(lp).all()
        assert (tok >= 0).all() and (tok < V).all()


@pytest.mark.parametrize("Hq,Hkv", [(28, 4), (12, 2)])
def test_tcgen05_attention_matches_mma_sync_and_reference(Hq, Hkv):
    """The tcgen05 forward (two ping-ponging query tiles per CTA) vs the mma.sync kernel
    and the fp32 reference on a random tree."""
    mode = 2
    rng = np.random.default_rng(13)
    torch.manual_seed(13)
    D = 128
    T, cu_q, cu_k, keys = _tree_plan(rng, n_nodes=10)
    plan = ops.AttnPlan.build(cu_q, cu_k, keys, dev)
    qkv = (torch.randn(T, (Hq + 2 * Hkv) * D, device=dev) * 0.5).bfloat16()
    q, k, v = qkv[:, : Hq * D], qkv[:, Hq * D: (Hq + Hkv) * D], qkv[:, (Hq + Hkv) * D:]
    o_tc, lse_tc = ops.ext().attn_fwd(q, k, v, plan.cu_q, plan.cu_k, plan.key_idx, plan.tiles_for(mode), Hq, Hkv, D,
                                      D ** -0.5, True, True, mode)
    o_ms, lse_ms = ops.ext().attn_fwd(q, k, v, plan.cu_q, plan.cu_k, plan.key_idx, plan.fwd_tiles, Hq, Hkv, D,
                                      D ** -0.5, True, True, 0)
    torch.cuda.synchronize()
    ops.check_status(0)
    x = qkv.float().cpu()
    orf, lrf = ref.gather_attention(x[:, : Hq * D].reshape(T, Hq, D), x[:, Hq * D: (Hq + Hkv) * D].reshape(T, Hkv, D),
                                    x[:, (Hq + Hkv) * D:].reshape(T, Hkv, D), cu_q, cu_k, torch.from_numpy(keys),
                                    D ** -0.5)
    assert rel_err(o_tc.cpu(), orf.reshape(T, Hq * D)) < 2e-2
    assert rel_err(o_tc, o_ms) < 2e-2
    assert torch.allclose(lse_tc.cpu(), lrf.float(), atol=2e-2)


@pytest.mark.parametrize("shuffle", [False, True])
def test_two_tile_attention_long_sequences(shuffle):
    """Two-tile forward on long sequences (several 256-row CTAs, the ragged last one) with
    keys in path order (TMA row boxes) or shuffled (cp.async gathers), against fp32."""
    rng = np.random.default_rng(21)
    torch.manual_seed(21)
    Hq, Hkv, D = 8, 2, 128
    pre, lens = 700, [900, 333, 1]
    T = pre + sum(lens)
    perm = rng.permutation(T).astype(np.int32) if shuffle else np.arange(T, dtype=np.int32)
    keys, cu_q, cu_k, qrows = [], [0], [0], []
    a = pre
    for n in lens:
        keys += list(perm[:pre]) + list(perm[a:a + n])
        qrows += list(range(a, a + n))
        cu_q.append(cu_q[-1] + n)
        cu_k.append(len(keys))
        a += n
    keys = np.asarray(keys, dtype=np.int32)
    plan = ops.AttnPlan.build(cu_q, cu_k, keys, dev)
    kv = (torch.randn(T, 2 * Hkv * D, device=dev) * 0.5).bfloat16()
    q = (torch.randn(cu_q[-1], Hq * D, device=dev) * 0.5).bfloat16()
    k, v = kv[:, : Hkv * D], kv[:, Hkv * D:]
    o, lse = ops.ext().attn_fwd(q, k, v, plan.cu_q, plan.cu_k, plan.key_idx, plan.tiles_for(2), Hq, Hkv, D,
                                D ** -0.5, True, True, 2)
    torch.cuda.synchronize()
    ops.check_status(0)
    orf, lrf = ref.gather_attention(q.float().cpu().reshape(-1, Hq, D), k.float().cpu().reshape(T, Hkv, D),
                                    v.float().cpu().reshape(T, Hkv, D), cu_q, cu_k, torch.from_numpy(keys), D ** -0.5)
    assert rel_err(o.cpu(), orf.reshape(-1, Hq * D)) < 2e-2
    assert torch.allclose(lse.cpu(), lrf.float(), atol=2e-2)


def test_persistent_decode_matches_splitk():
    torch.manual_seed(14)
    B, Hq, Hkv, D = 64, 28, 4, 128
    slots = 20000
    kc = torch.randn(slots, Hkv * D, device=dev).bfloat16()
    vc = torch.randn(slots, Hkv * D, device=dev).bfloat16()
    lens = torch.randint(1, 3000, (B,))
    ip = torch.zeros(B + 1, dtype=torch.int32)
    ip[1:] = torch.cumsum(lens, 0)
    idx = torch.randint(0, slots, (int(ip[-1]),), dtype=torch.int32, device=dev)
    q = torch.randn(B, Hq * D, device=dev).bfloat16()
    ipd = ip.to(dev)
    for splits in (1, 3, 8):
        a = ops.DecodeAttention(Hq, Hkv, D, B, splits, dev, persistent=True)(q, kc, vc, ipd, idx)
        b = ops.DecodeAttention(Hq, Hkv, D, B, splits, dev, persistent=False)(q, kc, vc, ipd, idx)
        assert rel_err(a, b) < 1e-2


@pytest.mark.gpu
@pytest.mark.parametrize("use_tc", [False, True])
def test_shared_prefix_decode_matches_persistent(use_tc):
    """Rows sharing a task prefix and a planner segment (DAG solver stage) plus unshared
    rows: the shared-prefix kernel equals the per-row kernel; dynamic lengths advance."""
    from test_decode_plan import dag_rows

    torch.manual_seed(15)
    Hq, Hkv, D = 28, 4, 128
    rows, ctx = dag_rows(n_inst=4, per=8, pre=700, plan=300, own=120)
    rows += [np.arange(200000, 200000 + 333), np.arange(210000, 210000 + 65)]
    ctx = np.r_[ctx, 300, 30]
    B = 40
    n = len(rows)
    slots = 220000
    kc = torch.randn(slots, Hkv * D, device=dev).bfloat16()
    vc = torch.randn(slots, Hkv * D, device=dev).bfloat16()
    starts = np.cumsum([0] + [len(r) for r in rows[:-1]]).astype(np.int32)
    idx = torch.from_numpy(np.concatenate(rows).astype(np.int32)).to(dev)
    final = np.asarray([len(r) for r in rows])
    q = torch.randn(B, Hq * D, device=dev).bfloat16()
    sd = ops.SharedDecode(Hq, Hkv, D, B, dev, use_tc=use_tc)
    assert sd.plan(rows, starts, ctx, final, B)
    assert sd.stats["shared_segments"] > 0
    pd = ops.DecodeAttention(Hq, Hkv, D, B, 4, dev, persistent=True)
    st = torch.zeros(B, dtype=torch.int32, device=dev)
    st[:n] = torch.from_numpy(starts).to(dev)
    for shrink in (20, 0):  # an earlier decode step (shorter own parts), then the full lengths
        ln = torch.zeros(B, dtype=torch.int32, device=dev)
        ln[:n] = torch.from_numpy(final - shrink).to(dev)
        a = sd(q, kc, vc, idx, ln)
        b = pd(q, kc, vc, st, idx, kv_len=ln)
        torch.cuda.synchronize()
        ops.check_status(0)
        assert rel_err(a[:n], b[:n]) < 1e-2
        assert float(a[n:].float().abs().max()) == 0.0


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K", [(16, 4608, 3584), (128, 3584, 18944), (256, 3584, 3584), (200, 512, 1024),
                                   (136, 2048, 4096), (232, 37888, 512), (256, 37888, 3584)])
def test_splitk_decode_gemm(M, N, K):
    """Decode-sized GEMMs: split-K (fp32 partials + finish with bias/residual) and, for
    128 < M <= 256, two M-tiles per CTA (with and without split-K)."""
    torch.manual_seed(16)
    a = (torch.randn(M, K, device=dev) * 0.5).bfloat16()
    w = (torch.randn(N, K, device=dev) * 0.02).bfloat16()
    b = (torch.randn(N, device=dev) * 0.1).bfloat16()
    r = torch.randn(M, N, device=dev).bfloat16()
    out = ops.gemm(a, w, bias=b, residual=r)
    torch.cuda.synchronize()
    ops.check_status(0)
    ref_ = a.float() @ w.float().t() + b.float() + r.float()
    assert rel_err(out, ref_) < 1e-2


@pytest.mark.gpu
@pytest.mark.parametrize("M", [144, 256])
def test_two_mtile_gemm_matches_one_mtile(M, monkeypatch):
    """MT = 2 (both M-blocks in one CTA) gives the same sums as the one-M-tile launch."""
    torch.manual_seed(17)
    a = (torch.randn(M, 3584, device=dev) * 0.5).bfloat16()
    w = (torch.randn(37888, 3584, device=dev) * 0.02).bfloat16()
    two = ops.gemm(a, w)
    monkeypatch.setenv("OCTO_GEMM_MT", "1")
    one = ops.gemm(a, w)
    torch.cuda.synchronize()
    ops.check_status(0)
    assert torch.equal(one, two)


def _bwd_both(q, k, v, plan, Hq, Hkv, D, seed):
    """(dq, dk, dv) of the tcgen05 and the mma.sync backward kernels on the same inputs."""
    torch.manual_seed(seed)
    T = q.shape[0]
    o, lse = ops.ext().attn_fwd(q, k, v, plan.cu_q, plan.cu_k, plan.key_idx, plan.tiles_for(2), Hq, Hkv, D,
                                D ** -0.5, True, True, 2)
    do = (torch.randn_like(o.float()) * 0.5).bfloat16()
    out = []
    for tc in (1, 0):
        dk = torch.zeros(k.shape[0], Hkv * D, dtype=torch.float32, device=dev)
        dv = torch.zeros_like(dk)
        dq = ops.ext().attn_bwd(q, k, v, o, do, lse, plan.cu_q, plan.cu_k, plan.key_idx,
                                plan.dq_tiles_tc if tc else plan.dq_tiles, plan.kv_tiles_tc if tc else plan.kv_tiles,
                                dk, dv, Hq, Hkv, D, D ** -0.5, True, tc)
        out.append((dq, dk, dv))
    torch.cuda.synchronize()
    ops.check_status(0)
    return out


@pytest.mark.parametrize("Hq,Hkv", [(28, 4), (12, 2)])
def test_tcgen05_attention_backward_tree(Hq, Hkv):
    """tcgen05 backward (dq kernel + dkv kernel) vs the mma.sync kernels on a random tree."""
    rng = np.random.default_rng(31)
    torch.manual_seed(31)
    D = 128
    T, cu_q, cu_k, keys = _tree_plan(rng, n_nodes=10)
    plan = ops.AttnPlan.build(cu_q, cu_k, keys, dev)
    qkv = (torch.randn(T, (Hq + 2 * Hkv) * D, device=dev) * 0.5).bfloat16()
    q, k, v = qkv[:, : Hq * D], qkv[:, Hq * D: (Hq + Hkv) * D], qkv[:, (Hq + Hkv) * D:]
    (a, b) = _bwd_both(q, k, v, plan, Hq, Hkv, D, 32)
    for x, y in zip(a, b):
        assert rel_err(x.float(), y.float()) < 2e-2


@pytest.mark.parametrize("shuffle", [False, True])
def test_tcgen05_attention_backward_long(shuffle):
    """Long sequences sharing a prefix (key rows in several lists: fp32 scatter-adds), keys
    consecutive (TMA boxes) or shuffled (cp.async gathers)."""
    rng = np.random.default_rng(33)
    Hq, Hkv, D = 8, 2, 128
    pre, lens = 700, [900, 333, 1]
    T = pre + sum(lens)
    perm = rng.permutation(T).astype(np.int32) if shuffle else np.arange(T, dtype=np.int32)
    keys, cu_q, cu_k = [], [0], [0]
    a = pre
    for n in lens:
        keys += list(perm[:pre]) + list(perm[a:a + n])
        cu_q.append(cu_q[-1] + n)
        cu_k.append(len(keys))
        a += n
    plan = ops.AttnPlan.build(cu_q, cu_k, np.asarray(keys, dtype=np.int32), dev)
    torch.manual_seed(34)
    kv = (torch.randn(T, 2 * Hkv * D, device=dev) * 0.5).bfloat16()
    q = (torch.randn(cu_q[-1], Hq * D, device=dev) * 0.5).bfloat16()
    (a_, b_) = _bwd_both(q, kv[:, : Hkv * D], kv[:, Hkv * D:], plan, Hq, Hkv, D, 35)
    for x, y in zip(a_, b_):
        assert rel_err(x.float(), y.float()) < 2e-2


@pytest.mark.parametrize("M", [16, 200, 256, 320])
def test_fused_decode_finishes_match_unfused(M):
    """gemm_res_norm / gemm_qkv_rope (split-K finish fused with residual + RMSNorm, and with
    bias + rotary + KV write) against the separate ops; M = 320 takes the unfused fallback."""
    from octopus_b200.ops import serve as sv

    torch.manual_seed(40 + M)
    H, Hq, Hkv, D = 3584, 28, 4, 128
    a = (torch.randn(M, H, device=dev) * 0.5).bfloat16()
    w = (torch.randn(H, H, device=dev) * 0.02).bfloat16()
    res = torch.randn(M, H, device=dev).bfloat16()
    nw = (torch.rand(H, device=dev) + 0.5).bfloat16()
    x, h = ops.ext().gemm_res_norm(a, w, res, nw, 1e-6, False, None)
    x_ref = ops.gemm(a, w, residual=res)
    h_ref = sv.rms(x_ref, nw, 1e-6, False)
    assert rel_err(x.float(), x_ref.float()) < 1e-2
    assert rel_err(h.float(), h_ref.float()) < 1e-2
    wq = (torch.randn((Hq + 2 * Hkv) * D, H, device=dev) * 0.02).bfloat16()
    bq = (torch.randn((Hq + 2 * Hkv) * D, device=dev) * 0.1).bfloat16()
    pos = torch.randint(0, 30000, (M,), device=dev, dtype=torch.int32)
    slots = torch.randperm(4 * M, device=dev)[:M].long()
    slots[::7] = -1  # unwritten rows
    kc, vc = (torch.zeros(4 * M, Hkv * D, device=dev).bfloat16() for _ in range(2))
    kc2, vc2 = kc.clone(), vc.clone()
    q = ops.ext().gemm_qkv_rope(a, wq, bq, pos, 1e6, Hq, Hkv, D, slots, kc, vc)
    qkv = ops.gemm(a, wq, bias=bq)
    sv.rope_(qkv, pos, Hq, Hkv, D, 1e6)
    sv.kv_write(qkv, Hq, Hkv, D, slots, kc2, vc2)
    torch.cuda.synchronize()
    ops.check_status(0)
    assert rel_err(q.float(), qkv[:, : Hq * D].float()) < 1e-2
    assert rel_err(kc.float(), kc2.float()) < 1e-2 and rel_err(vc.float(), vc2.float()) < 1e-2
