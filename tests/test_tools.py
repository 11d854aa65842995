"""Probes on CPU: tree vs alone vs packed, mount parity (with gradients through the
mount), and the embedding table's gradient (regression: the table must be trained)."""
import numpy as np
import torch

from octopus_b200.tools import mount_check, tree_check


def test_tree_check_matches_alone_and_packed():
    out = tree_check.run(n_seqs=3, prefix=60, tail=40)
    assert out["packed_vs_alone_max"] < 1e-4
    assert out["tree_total_vs_alone"] < 1e-2
    assert out["grad_rel_l2_tree_vs_packed"] < 1e-4
    assert out["tree_pairs"] < out["positions"]


def test_mount_check_parity_and_backward():
    out = mount_check.run(points=2, backward=True)
    assert out["mounted_max_gap"] < 1e-4 and out["plain_max_gap"] < 1e-4
    assert out["grads_finite"] and out["mounted_token_grad_min"] > 0


def test_embedding_gets_gradient():
    from octopus_b200.models.config import get_config
    from octopus_b200.models.decoder import FlatLayout, Weights, forward_tree, init_flat
    from octopus_b200.rl.actor import build_microbatch

    cfg = get_config("tiny")
    lay = FlatLayout(cfg)
    grad = torch.zeros(lay.total)
    w = Weights(cfg, init_flat(cfg, lay, "cpu", dtype=torch.float32, seed=0, std=0.05), lay, grad)
    toks = np.random.default_rng(0).integers(1, cfg.vocab_size, 24)
    mb = build_microbatch(toks, [0, 24], None, np.ones(24, np.float32), np.ones(24, np.float32),
                          np.zeros(24, np.float32), pad_to=8)
    d = mb.to_device("cpu")
    lp, _ = forward_tree(w, d.batch, ckpt=True)
    lp.sum().backward()
    assert float(w["embed"].main_grad[torch.as_tensor(toks[:-1])].norm()) > 0


def test_act_gpu_bench_settings_agree():
    """Every memory setting gives the first one's gradients (float64 on CPU), LoRA too."""
    from octopus_b200.tools.act_gpu_bench import parse_setting, run

    assert parse_setting("chunk:64+tile:16") == {"ckpt_block": 1, "act_gpu_bytes": None, "chunk_tokens": 64,
                                                   "seq_tile": 16}
    for lora in (0, 4):
        rows = run(["layer", "block:2", "chunk:40", "tile:16", "chunk:40+tile:8"], 150, preset="tiny", layers=2,
                   lora=lora, group=3, device="cpu")
        assert len(rows) == 5 and rows[0]["tree_tokens"] > 0
        assert all(r["grad_rel_l2"] < 1e-9 for r in rows), rows
