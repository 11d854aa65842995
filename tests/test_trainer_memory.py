"""Trainer memory features on CPU: block checkpointing and host-resident saved activations
give the same loss and gradients as per-layer checkpointing; the pinned slab carves
aligned pieces and grows; host activations refuse to run without checkpointing."""
import numpy as np
import pytest
import torch

from octopus_b200.models.config import get_config
from octopus_b200.models.decoder import FlatLayout, Weights, forward_tree, init_flat
from octopus_b200.rl.actor import build_microbatch
from octopus_b200.utils.pinned_slab import HostActivations, PinnedSlab, check_checkpointing


def _setup(layers=4):
    cfg = get_config("tiny", layers=layers)
    lay = FlatLayout(cfg)
    grad = torch.zeros(lay.total, dtype=torch.float64)
    w = Weights(cfg, init_flat(cfg, lay, "cpu", dtype=torch.float64, seed=1, std=0.05), lay, grad)
    rng = np.random.default_rng(0)
    toks = rng.integers(1, cfg.vocab_size, 64)
    mb = build_microbatch(np.r_[toks, toks[:40], rng.integers(1, cfg.vocab_size, 20)], [0, 64, 124], None,
                          np.ones(124, np.float32), rng.normal(size=124).astype(np.float32), np.zeros(124, np.float32),
                          pad_to=8)
    return w, grad, mb.to_device("cpu")


def _run(w, grad, d, **kw):
    grad.zero_()
    lp, _ = forward_tree(w, d.batch, ckpt=True, **kw)
    (lp * d.adv.to(lp.dtype) * d.w.to(lp.dtype)).sum().backward()
    return lp.detach().clone(), grad.clone()


def test_block_checkpoint_matches_layer_checkpoint():
    w, grad, d = _setup()
    lp1, g1 = _run(w, grad, d)
    for k in (2, 3):
        lp2, g2 = _run(w, grad, d, ckpt_block=k)
        assert torch.allclose(lp1, lp2) and torch.allclose(g1, g2, rtol=1e-9, atol=1e-12)


def test_host_activations_context_and_slab():
    w, grad, d = _setup()
    lp1, g1 = _run(w, grad, d)
    with HostActivations(gpu_budget=0, min_bytes=0):
        lp = forward_tree(w, d.batch, ckpt=True)[0]
    grad.zero_()
    (lp * d.adv.to(lp.dtype) * d.w.to(lp.dtype)).sum().backward()
    assert torch.allclose(lp.detach(), lp1) and torch.allclose(grad, g1, rtol=1e-9, atol=1e-12)
    s = PinnedSlab()
    s.reserve(4096)
    a, b = s.take(100), s.take(100)
    assert a is not None and b is not None and (b.data_ptr() - a.data_ptr()) % 512 == 0
    assert s.take(1 << 20) is None
    s.release()
    assert s.take(4000) is not None
    with pytest.raises(ValueError):
        check_checkpointing(False, HostActivations(0))


def test_sequence_tiles_match_whole_layer():
    """o-projection + MLP in checkpointed row tiles: same logprobs and gradients as the
    untiled layer (tiles of 8 and 24 rows, with block checkpointing too)."""
    w, grad, d = _setup()
    lp1, g1 = _run(w, grad, d)
    for kw in ({"seq_tile": 8}, {"seq_tile": 24}, {"seq_tile": 16, "ckpt_block": 2}):
        lp2, g2 = _run(w, grad, d, **kw)
        assert torch.allclose(lp1, lp2, rtol=1e-12, atol=1e-12) and torch.allclose(g1, g2, rtol=1e-9, atol=1e-12)
