"""Chunk-major training on CPU (float64): a prefix tree with a mount, run in chunks of a few
rows, gives the same logprobs, entropies and parameter gradients as the whole-tree forward;
the plan keeps exactly the rows later chunks read and orders chunks after their keys."""
import numpy as np
import pytest
import torch

from octopus_b200.models.config import get_config
from octopus_b200.models.decoder import FlatLayout, Weights, forward_tree, init_flat
from octopus_b200.rl.actor import build_microbatch
from octopus_b200.rl.chunk_major import ChunkPlan, chunk_major_forward


def _setup(layers=3, mounts=True):
    cfg = get_config("tiny", layers=layers)
    lay = FlatLayout(cfg)
    grad = torch.zeros(lay.total, dtype=torch.float64)
    w = Weights(cfg, init_flat(cfg, lay, "cpu", dtype=torch.float64, seed=2, std=0.05), lay, grad)
    rng = np.random.default_rng(3)
    a = rng.integers(1, cfg.vocab_size, 50)
    b = np.r_[a[:30], rng.integers(1, cfg.vocab_size, 25)]      # shares 30 tokens with a
    c = rng.integers(1, cfg.vocab_size, 40)                       # mounts a[10:20] at its row 15
    flat = np.r_[a, b, c]
    cu = [0, 50, 105, 145]
    m = {2: [(15, 0, 10, 20)]} if mounts else None
    n = len(flat)
    mb = build_microbatch(flat, cu, m, np.ones(n, np.float32), rng.normal(size=n).astype(np.float32),
                          np.zeros(n, np.float32), pad_to=8)
    return w, grad, mb


def _loss(lp, ent, d):
    return (lp * d.adv.to(lp.dtype) * d.w.to(lp.dtype)).sum() + 0.1 * (ent * d.w.to(ent.dtype)).sum()


@pytest.mark.parametrize("tokens", [8, 16, 40, 1000])
@pytest.mark.parametrize("mounts", [False, True])
def test_chunk_major_matches_whole_tree(tokens, mounts):
    w, grad, mb = _setup(mounts=mounts)
    d = mb.to_device("cpu")
    grad.zero_()
    lp, ent = forward_tree(w, d.batch, ckpt=True)
    _loss(lp, ent, d).backward()
    g_ref = grad.clone()
    grad.zero_()
    lp2, ent2 = chunk_major_forward(w, mb, tokens)
    _loss(lp2, ent2, d).backward()
    assert torch.allclose(lp2, lp.detach(), rtol=1e-9, atol=1e-10)
    assert torch.allclose(ent2, ent.detach(), rtol=1e-9, atol=1e-10)
    assert torch.allclose(grad, g_ref, rtol=1e-7, atol=1e-10), float((grad - g_ref).abs().max())


def test_plan_keeps_only_rows_read_later():
    _, _, mb = _setup(mounts=True)
    plan = ChunkPlan(mb, 16)
    seen = set()
    for c, ch in enumerate(plan.chunks):
        assert len(ch.rows) <= 16
        assert (ch.ext_slots < plan.n_kept).all()
        # what a chunk reads from earlier chunks lives in earlier chunks' slot blocks
        assert all(s < ch.own_lo for s in ch.ext_slots)
        seen |= set(ch.ext_slots.tolist())
    assert seen == set(range(plan.n_kept))  # every kept slot is read by some chunk
    assert sum(len(ch.rows) for ch in plan.chunks) == len(mb.tokens) - (len(mb.tokens) - mb.cu_q[-1])


def test_actor_chunk_major_knob_matches_default():
    """Actor.set_memory(chunk_tokens=...) routes larger micro-batches through chunk-major
    with the same gradients as the whole-tree path."""
    from octopus_b200.rl.actor import Actor

    cfg = get_config("tiny", layers=2)
    _, _, mb = _setup(layers=2)
    grads = []
    for ct in (0, 24):
        actor = Actor(cfg, "cpu", seed=5, dtype=torch.float64)
        actor.set_memory(chunk_tokens=ct)
        actor.zero_grad()
        st = actor.forward_backward([mb])
        grads.append((actor.grad.clone(), float(st["loss"])))
    assert abs(grads[0][1] - grads[1][1]) < 1e-9
    assert torch.allclose(grads[0][0], grads[1][0], rtol=1e-7, atol=1e-10)


@pytest.mark.gpu
def test_chunk_major_gpu_matches_whole_tree():
    """bf16 on the sm_100a kernels (7B layer shapes, 2 layers): chunk-major with 96-row chunks
    against the whole-tree forward / backward."""
    dev = torch.device("cuda", 0)
    cfg = get_config("qwen2.5-7b", layers=2)
    lay = FlatLayout(cfg)
    grad = torch.zeros(lay.total, dtype=torch.float32, device=dev)
    w = Weights(cfg, init_flat(cfg, lay, dev, seed=4), lay, grad)
    _, _, mb = _setup(mounts=True)
    mb.tokens = np.minimum(mb.tokens, cfg.vocab_size - 1)
    d = mb.to_device(dev)
    lp, ent = forward_tree(w, d.batch, ckpt=True)
    _loss(lp, ent, d).backward()
    g_ref = grad.clone()
    grad.zero_()
    lp2, ent2 = chunk_major_forward(w, mb, 96)
    _loss(lp2, ent2, d).backward()
    torch.cuda.synchronize()
    rel = lambda a, b: float((a.float() - b.float()).norm() / (b.float().norm() + 1e-12))  # noqa: E731
    assert rel(lp2, lp.detach()) < 1e-2 and rel(ent2, ent.detach()) < 1e-2
    assert rel(grad, g_ref) < 3e-2


def _hybrid_setup(kind, mounts):
    from octopus_b200.models.hybrid import HybridConfig, HybridWeights

    base = get_config("tiny", layers=4, vocab_size=512)
    hw = HybridWeights(HybridConfig(base, kind=kind, pattern="LLAL", lin_heads=2, lin_dim=32), "cpu",
                       dtype=torch.float64, seed=4, std=0.05)
    rng = np.random.default_rng(5)
    root = rng.integers(1, 512, 21)
    a = np.r_[root, rng.integers(1, 512, 13)]
    b = np.r_[root, rng.integers(1, 512, 18)]
    c = np.r_[a, rng.integers(1, 512, 9)]  # below a's node: depth 2
    e = rng.integers(1, 512, 17)            # mounts a[3:9] at its row 6
    seqs = [a, b, c, e]
    flat = np.concatenate(seqs)
    cu = np.r_[0, np.cumsum([len(x) for x in seqs])]
    n = len(flat)
    m = {3: [(6, 0, 3, 9)]} if mounts else None
    mb = build_microbatch(flat, cu, m, np.ones(n, np.float32), rng.normal(size=n).astype(np.float32),
                          np.zeros(n, np.float32), pad_to=8)
    return hw, mb


def _hybrid_grads(hw):
    return torch.cat([hw.grad] + [t.main_grad.reshape(-1) for t in hw.t.values()] +
                     [p.grad.reshape(-1) for p in hw.fp32.values()])


def _hybrid_zero(hw):
    hw.grad.zero_()
    for t in hw.t.values():
        t.main_grad.zero_()
    for p in hw.fp32.values():
        p.grad = None


@pytest.mark.parametrize("tokens", [8, 13, 24, 1000])
@pytest.mark.parametrize("kind,mounts", [("gdn", False), ("gdn", True), ("gla", False)])
def test_hybrid_chunk_major_matches_whole_tree(kind, mounts, tokens):
    """Linear layers keep states and conv input rows across chunks: chunks of a few rows
    (nodes split into parts, parents in earlier chunks) give the whole-tree logprobs and
    every parameter gradient (dense, linear-layer and fp32 gate / conv parameters)."""
    from octopus_b200.models.hybrid import hybrid_forward

    hw, mb = _hybrid_setup(kind, mounts)
    assert mb.nodes[:, 3].max() >= 2
    d = mb.to_device("cpu")
    _hybrid_zero(hw)
    lp, ent = hybrid_forward(hw, d.batch)
    _loss(lp, ent, d).backward()
    g_ref = _hybrid_grads(hw).clone()
    _hybrid_zero(hw)
    lp2, ent2 = chunk_major_forward(hw, mb, tokens)
    _loss(lp2, ent2, d).backward()
    assert torch.allclose(lp2, lp.detach(), rtol=1e-9, atol=1e-10)
    assert torch.allclose(ent2, ent.detach(), rtol=1e-9, atol=1e-10)
    g = _hybrid_grads(hw)
    assert torch.allclose(g, g_ref, rtol=1e-7, atol=1e-10), float((g - g_ref).abs().max())


@pytest.mark.gpu
def test_hybrid_chunk_major_gpu_matches_whole_tree():
    """bf16 on the sm_100a kernels (7B attention shapes, GDN layers with 2 heads of 128):
    hybrid chunk-major with 16-row chunks against the whole-tree forward / backward."""
    from octopus_b200.models.hybrid import HybridConfig, HybridWeights, hybrid_forward

    dev = torch.device("cuda", 0)
    _, mb = _hybrid_setup("gdn", True)
    hw = HybridWeights(HybridConfig(get_config("qwen2.5-7b", layers=4), kind="gdn", pattern="LLAL", lin_heads=2,
                                    lin_dim=128), dev, dtype=torch.bfloat16, seed=4)
    d = mb.to_device(dev)
    _hybrid_zero(hw)
    lp, ent = hybrid_forward(hw, d.batch)
    _loss(lp, ent, d).backward()
    g_ref = _hybrid_grads(hw).clone()
    _hybrid_zero(hw)
    lp2, ent2 = chunk_major_forward(hw, mb, 16)
    _loss(lp2, ent2, d).backward()
    torch.cuda.synchronize()
    rel = lambda a, b: float((a.float() - b.float()).norm() / (b.float().norm() + 1e-12))  # noqa: E731
    assert rel(lp2, lp.detach()) < 1e-2 and rel(ent2, ent.detach()) < 1e-2
    assert rel(_hybrid_grads(hw), g_ref) < 3e-2
