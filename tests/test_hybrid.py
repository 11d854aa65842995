"""Hybrid (linear recurrence + attention) decoder over prefix trees on CPU, fp64: the tree
forward (conv context from ancestors, level-by-level states from parents) scores every
sequence exactly as running it alone, for the gated-DeltaNet and GLA (Mamba-2) forms;
gradients of a weighted loss match the per-sequence sum; unknown stateful families raise."""
import numpy as np
import pytest
import torch

from octopus_b200.models.config import get_config
from octopus_b200.models.hybrid import HybridConfig, HybridWeights, family_kind, hybrid_forward
from octopus_b200.rl.actor import build_microbatch


def _hw(kind):
    base = get_config("tiny", layers=4, vocab_size=512)
    return HybridWeights(HybridConfig(base, kind=kind, pattern="LLLA", lin_heads=4, lin_dim=64), "cpu",
                         dtype=torch.float64, seed=2, std=0.05)


def _seqs(rng, V):
    root = rng.integers(1, V, 20)
    a = np.r_[root, rng.integers(1, V, 7)]
    b = np.r_[root, rng.integers(1, V, 11)]
    c = np.r_[a, rng.integers(1, V, 5)]  # forks below a's node: depth 2
    return [a, b, c]


@pytest.mark.parametrize("kind", ["gdn", "gla"])
def test_tree_equals_alone(kind):
    hw = _hw(kind)
    rng = np.random.default_rng(0)
    seqs = _seqs(rng, 512)
    flat = np.concatenate(seqs)
    cu = np.r_[0, np.cumsum([len(s) for s in seqs])]
    n = len(flat)
    mb = build_microbatch(flat, cu, None, np.ones(n, np.float32), np.zeros(n, np.float32), np.zeros(n, np.float32),
                          pad_to=8)
    assert mb.nodes[:, 3].max() >= 2  # really a tree
    d = mb.to_device("cpu")
    with torch.no_grad():
        lp_tree, _ = hybrid_forward(hw, d.batch)
        tot_tree = float((lp_tree * d.w.double()).sum())
        tot_alone = 0.0
        for s in seqs:
            m1 = build_microbatch(s, [0, len(s)], None, np.ones(len(s), np.float32), np.zeros(len(s), np.float32),
                                  np.zeros(len(s), np.float32), pad_to=8)
            d1 = m1.to_device("cpu")
            lp1, _ = hybrid_forward(hw, d1.batch)
            tot_alone += float((lp1 * d1.w.double()).sum())
    assert abs(tot_tree - tot_alone) < 1e-8 * max(1.0, abs(tot_alone))


def test_tree_gradients_equal_flat_sum():
    hw = _hw("gdn")
    rng = np.random.default_rng(1)
    seqs = _seqs(rng, 512)

    def loss_of(idx_groups):
        for p in [*hw.fp32.values()]:
            p.grad = None
        hw.grad.zero_()
        for t in hw.t.values():
            t.main_grad.zero_()
        total = 0.0
        for idx in idx_groups:
            flat = np.concatenate([seqs[i] for i in idx])
            cu = np.r_[0, np.cumsum([len(seqs[i]) for i in idx])]
            n = len(flat)
            wts = np.concatenate([np.linspace(-1, 1, len(seqs[i])) for i in idx]).astype(np.float32)
            mb = build_microbatch(flat, cu, None, np.ones(n, np.float32), wts, np.zeros(n, np.float32), pad_to=8)
            d = mb.to_device("cpu")
            lp, _ = hybrid_forward(hw, d.batch)
            loss = (lp * d.adv.double() * d.w.double()).sum()
            loss.backward()
            total += float(loss.detach())
        grads = torch.cat([hw.grad] + [t.main_grad.reshape(-1) for t in hw.t.values()] +
                          [p.grad.reshape(-1) for p in hw.fp32.values()])
        return total, grads

    l1, g1 = loss_of([[0, 1, 2]])
    l2, g2 = loss_of([[0], [1], [2]])
    # (pair advantages are fp32 averages over the positions sharing a pair: ~1e-7 relative)
    assert abs(l1 - l2) < 1e-6 * abs(l2)
    assert float((g1 - g2).norm() / g2.norm()) < 1e-6


def test_families():
    assert family_kind("qwen3_5") == "gdn" and family_kind("granitemoehybrid") == "gla"
    with pytest.raises(ValueError):
        family_kind("jamba")
