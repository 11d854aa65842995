"""KV-pool pressure on the CPU engine (fp64): instead of failing with OutOfKV, the engine
spills least-recently-used cursors (drops their KV, keeps their recipe) and rebuilds a
spilled cursor or mount source when a request continues or mounts it.  A random workload
of prompts, continuations, mounts (K1 / K2 / K3) and releases on a small pool must give
the same tokens and logprobs as the same workload on a pool that never spills, with pool
balance (every slot free again after the cursors are released) and no double free (the
native pool raises on one)."""
import numpy as np
import pytest
import torch

from octopus_b200.serving.engine import CursorNotFound, GenInput
from test_engine_cpu import tiny_engine


def _pair(small_slots):
    _, _, big = tiny_engine(torch.float64)
    cfg, _, small = tiny_engine(torch.float64)
    from octopus_b200.serving.engine import Engine

    small = Engine(cfg, small.w, kv_slots=small_slots, max_batch=16, device="cpu")
    return cfg, big, small


def test_spilled_cursor_and_mount_source_are_rebuilt_exactly():
    cfg, big, small = _pair(700)
    rng = np.random.default_rng(0)
    a_prompt = rng.integers(1, cfg.vocab_size, 120).tolist()
    outs = {}
    for name, eng in (("big", big), ("small", small)):
        a = eng.generate([GenInput(a_prompt, max_new_tokens=20, rid=1, cursor_id="A")])[0]
        b = eng.generate([GenInput(rng_tokens(5, cfg), mount=[("A", 10, 90)], max_new_tokens=15, rid=2,
                                   cursor_id="B")])[0]
        # fill the pool with other work so that A and B get spilled on the small engine
        for k in range(4):
            eng.generate([GenInput(rng_tokens(100 + k, cfg, seed=k), max_new_tokens=30, rid=10 + k,
                                   cursor_id=f"F{k}")])
        c = eng.generate([GenInput(rng_tokens(7, cfg, seed=99), cursor="B", max_new_tokens=12, rid=3)])[0]
        d = eng.generate([GenInput(rng_tokens(6, cfg, seed=98), mount=[("A", 0, 50)], max_new_tokens=8, rid=4)])[0]
        outs[name] = (a, b, c, d)
    for x, y in zip(outs["big"], outs["small"]):
        assert x.output_ids == y.output_ids
        assert np.allclose(x.output_logprobs, y.output_logprobs, atol=1e-9)
    assert small.stats.get("spills", 0) > 0 and small.stats.get("rebuilds", 0) >= 1


def rng_tokens(n, cfg, seed=7):
    return np.random.default_rng(seed * 1000 + n).integers(1, cfg.vocab_size, n).tolist()


@pytest.mark.parametrize("seed", [0, 1])
def test_random_workload_matches_unpressured_pool(seed):
    cfg, big, small = _pair(900)
    free0 = {"big": big.pool.free_count(), "small": small.pool.free_count()}
    rng = np.random.default_rng(seed)
    live: list[str] = []
    sources: set[str] = set()  # mounted cursors stay alive (a spilled dependent rebuilds from them)
    for step in range(40):
        op = rng.choice(["new", "cont", "mount", "release"], p=[0.3, 0.3, 0.3, 0.1]) if live else "new"
        cid = f"c{step}"
        toks = rng.integers(1, cfg.vocab_size, int(rng.integers(3, 60))).tolist()
        max_new = int(rng.integers(1, 25))
        if op == "release":
            free = [c for c in live if c not in sources]
            if not free:
                continue
            victim = free[int(rng.integers(len(free)))]
            live.remove(victim)
            big.release_cursor(victim)
            small.release_cursor(victim)
            continue
        kw = {}
        if op == "cont":
            kw["cursor"] = live[int(rng.integers(len(live)))]
        if op == "mount":
            src = live[int(rng.integers(len(live)))]
            n = big.cursors.get(src).length
            a = int(rng.integers(0, max(1, n - 2)))
            b = int(rng.integers(a + 1, n))
            if (big.cursors.get(src).slots[a:b] < 0).any():
                continue  # rows without KV cannot be mounted
            kw["mount"] = [(src, a, b)]
            sources.add(src)
            kw["mount_rule"] = str(rng.choice(["K1", "K2", "K3"]))
        res = {}
        for name, eng in (("big", big), ("small", small)):
            res[name] = eng.generate([GenInput(toks, max_new_tokens=max_new, rid=step, cursor_id=cid, **kw)])[0]
        assert res["big"].output_ids == res["small"].output_ids, step
        assert np.allclose(res["big"].output_logprobs, res["small"].output_logprobs, atol=1e-9), step
        live.append(cid)
    assert small.stats.get("spills", 0) > 0
    for name, eng in (("big", big), ("small", small)):
        eng.reset()
        assert eng.pool.free_count() == free0[name], name


def test_rebuild_fails_alone_when_a_mount_source_is_gone():
    cfg, big, small = _pair(500)
    small.generate([GenInput(rng_tokens(100, cfg), max_new_tokens=10, cursor_id="S")])
    small.generate([GenInput(rng_tokens(4, cfg), mount=[("S", 0, 60)], max_new_tokens=10, cursor_id="R")])
    for k in range(4):
        small.generate([GenInput(rng_tokens(90, cfg, seed=k), max_new_tokens=30, cursor_id=f"F{k}")])
    assert small.cursors.peek("R").meta.get("spilled")
    small.release_cursor("S")
    with pytest.raises(CursorNotFound):
        small.generate([GenInput(rng_tokens(3, cfg), cursor="R", max_new_tokens=2)])
    # other requests still run
    assert len(small.generate([GenInput(rng_tokens(9, cfg), max_new_tokens=3)])[0].output_ids) == 3
