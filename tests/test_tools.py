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


def test_rollout_and_mount_load_run_on_the_engine():
    """rollout_load runs DAG rollouts with weight-version switches; mount_load runs fork
    pairs whose forced reads mount the sibling's own rows (tiny CPU engine)."""
    import io
    import json

    import torch

    from octopus_b200.envs.dag import DagConfig, MultiAgentDag
    from octopus_b200.models.config import get_config
    from octopus_b200.models.decoder import FlatLayout, Weights, init_flat
    from octopus_b200.serving.engine import Engine
    from octopus_b200.tools import mount_load, rollout_load

    cfg = get_config("tiny", vocab_size=512, layers=2)
    lay = FlatLayout(cfg)
    w = Weights(cfg, init_flat(cfg, lay, "cpu", dtype=torch.float32, seed=3, std=0.05), lay)
    eng = Engine(cfg, w, kv_slots=60000, max_batch=16, device="cpu")
    env = MultiAgentDag(cfg.vocab_size, DagConfig(instances=1, samples=2, prefix_len=32, turn_len=4, role_len=4))
    buf = io.StringIO()
    s = rollout_load.run(eng, env, rollouts=2, duration=600, switch=1e-9, out=buf)
    assert s["rollouts"] == 2 and s["generated_tokens"] > 0 and s["version_switches"] == 1
    assert len(buf.getvalue().splitlines()) == 2
    buf = io.StringIO()
    st = mount_load.run(eng, cfg.vocab_size, pairs=2, duration=600, turns=(6, 8), root=40, tool=12, reply=(3, 6),
                        mount=10, seed=1, out=buf)
    rows = [json.loads(x) for x in buf.getvalue().splitlines()]
    assert st["pairs"] == 2 and st["reads"] > 0 and st["mounted_tokens"] > 0 and st["not_found"] == 0
    assert any(r["kind"] == "read" and r["mounted"] > 0 for r in rows)


def test_prefix_flops_rules(tmp_path):
    """Analytic prefix-reuse FLOPs: a thread reuses its previous request, a branch its parent's
    latest, main's first nothing; the saving is 1 - reuse / no-reuse; logs are read from
    episode directories; hybrid presets count attention layers only in the quadratic term."""
    import json

    from octopus_b200.tools.prefix_flops import episode_flops, model_constants, run

    reqs = [{"thread": "main", "prompt_tokens": 100, "completion_tokens": 10},
            {"thread": "fork0/branch-0", "prompt_tokens": 130, "completion_tokens": 5},
            {"thread": "main", "prompt_tokens": 150, "completion_tokens": 20}]
    r = episode_flops(reqs, 1.0, 0.0)
    # reuse: main 100+10, branch (130-110)+5, main (150-110)+20 ; none: 110 + 135 + 170
    assert r["flops_reuse"] == 110 + 25 + 60 and r["flops_no_reuse"] == 110 + 135 + 170
    q = episode_flops(reqs[:1], 0.0, 1.0)
    assert q["flops_reuse"] == 100 * 100 / 2 + 10 * 100 + 10 * 10 / 2
    d = tmp_path / "ep"
    d.mkdir()
    (d / "requests.jsonl").write_text("".join(json.dumps(x) + "\n" for x in reqs))
    tot = run([str(tmp_path)], "tiny")
    assert tot["episodes"] == 1 and 0 < tot["saving"] < 1
    ct_d, ca_d = model_constants("tiny")
    ct_h, ca_h = model_constants("tiny-hybrid")
    assert ca_d > 0 and ca_h == 0 and ct_h > 0  # tiny-hybrid's two layers are both linear (pattern LLLA)
