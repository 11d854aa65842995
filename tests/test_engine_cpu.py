"""Engine cursor / mount / radix semantics and rollout-vs-trainer logprob parity (CPU, fp32)."""
import numpy as np
import pytest
import torch

from octopus_b200.envs.dag import DagConfig, MultiAgentDag, instance_microbatches
from octopus_b200.models.config import get_config
from octopus_b200.models.decoder import FlatLayout, Weights, forward_tree, init_flat
from octopus_b200.rl.actor import build_microbatch
from octopus_b200.serving.engine import CursorNotFound, Engine, GenInput


def tiny_engine(dtype=torch.float32, **kw):
    cfg = get_config("tiny", vocab_size=512, layers=2)
    lay = FlatLayout(cfg)
    flat = init_flat(cfg, lay, "cpu", dtype=dtype, seed=3, std=0.05)
    w = Weights(cfg, flat, lay)
    return cfg, w, Engine(cfg, w, kv_slots=20000, max_batch=16, device="cpu", **kw)


def test_generate_cursor_continuation_matches_full_prompt():
    cfg, w, eng = tiny_engine()
    rng = np.random.default_rng(0)
    prompt = rng.integers(1, cfg.vocab_size, 40).tolist()
    a = eng.generate([GenInput(prompt, max_new_tokens=6, cursor_id="a")])[0]
    delta = rng.integers(1, cfg.vocab_size, 5).tolist()
    b = eng.generate([GenInput(delta, cursor="a", max_new_tokens=4, cursor_id="b")])[0]
    cur_b = eng.cursors.get("b")
    full = prompt + a.output_ids + delta + b.output_ids
    assert cur_b.tokens.tolist() == full
    assert cur_b.positions.tolist() == list(range(len(full)))
    # the continuation's logprobs equal a fresh forward of the whole sequence
    mb = build_microbatch(np.asarray(full), [0, len(full)], None,
                          np.r_[np.zeros(len(full) - 4), np.ones(4)], np.zeros(len(full)), np.zeros(len(full)))
    d = mb.to_device("cpu")
    lp, _ = forward_tree(w, d.batch, ckpt=False)
    assert np.allclose(lp.detach().numpy(), b.output_logprobs, atol=1e-4)
    with pytest.raises(CursorNotFound):
        eng.generate([GenInput([1, 2], cursor="nope")])


def test_pool_balance_after_release():
    cfg, w, eng = tiny_engine()
    free0 = eng.pool.free_count()
    outs = eng.generate([GenInput(list(range(1, 30)), max_new_tokens=5, cursor_id=f"x{i}") for i in range(3)])
    eng.generate([GenInput([7, 8, 9], mount=[("x0", 0, 10), ("x1", 3, 12)], max_new_tokens=3, cursor_id="m")])
    for cid in ("x0", "x1", "x2", "m"):
        eng.release_cursor(cid)
    eng.reset()
    assert eng.pool.free_count() == free0
    assert eng.pool.check_invariants()
    del outs


def test_dag_rollout_logprobs_match_tree_trainer():
    """Rollout (cursors + zero-copy mounts + K2) and the prefix-tree trainer agree exactly."""
    cfg, w, eng = tiny_engine()
    env = MultiAgentDag(cfg.vocab_size, DagConfig(instances=2, samples=2, prefix_len=24, turn_len=6, role_len=3))
    ro = env.rollout(eng)
    mbs = instance_microbatches(ro, 10 ** 6, build_microbatch)
    assert len(mbs) == 1
    mb = mbs[0]
    d = mb.to_device("cpu")
    lp, _ = forward_tree(w, d.batch, ckpt=False)
    m = mb.pair_w > 0
    assert np.allclose(lp.detach().numpy()[m], mb.pair_behav[m], atol=2e-4)
    # every generated token is trained exactly once
    assert int(mb.pair_w.sum()) == ro.generated_tokens
    assert eng.pool.check_invariants()
