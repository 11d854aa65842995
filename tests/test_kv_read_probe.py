"""Mount position rules K1 / K2 / K3 and the cross-branch read probe on a tiny CPU engine:
K3 equals K2 where A's turn rows already sit at B's next positions, K1 equals K2 where they
sit below them, K3 relocation needs the rotary identity R(d) R(p) = R(p + d), every condition
runs, and no KV slot leaks."""
import numpy as np
import torch

from octopus_b200.ops import serve as sv
from octopus_b200.tools.kv_read_probe import CONDITIONS, report, run_probe, synthetic_probes
from test_engine_cpu import tiny_engine


def _probe(la, lb, lt=24, seed=0):
    rng = np.random.default_rng(seed)
    t = lambda n: rng.integers(1, 500, n).tolist()  # noqa: E731
    return {"a_prefix": t(la), "a_turns": t(lt), "b_prefix": t(lb), "question": t(6), "answer": t(4), "header": t(3)}


def test_k3_equals_k2_when_positions_coincide():
    cfg, w, eng = tiny_engine()
    r = run_probe(eng, _probe(40, 40), ("K2", "K3"))
    assert r["K2"]["output"] == r["K3"]["output"] and r["K2"]["first_pos"] == r["K3"]["first_pos"] == 40 + 24
    assert abs(r["K2"]["logprob"] - r["K3"]["logprob"]) < 1e-5


def test_k1_equals_k2_below_next_and_first_positions():
    cfg, w, eng = tiny_engine()
    r = run_probe(eng, _probe(10, 60), ("K1", "K2", "K3"))
    assert r["K1"]["output"] == r["K2"]["output"] and r["K1"]["first_pos"] == r["K2"]["first_pos"] == 60
    assert r["K3"]["first_pos"] == 60 + 24
    r = run_probe(eng, _probe(60, 10), ("K1", "K2"), tag="q")
    assert r["K1"]["first_pos"] == 10 and r["K2"]["first_pos"] == 60 + 24


def test_rotary_shift_composes():
    torch.manual_seed(0)
    k = torch.randn(5, 2 * 32, dtype=torch.float64)
    p = torch.tensor([0, 3, 17, 100, 5], dtype=torch.int32)
    d = torch.tensor([4, -3, 9, -100, 0], dtype=torch.int32)
    a, b = k.clone(), k.clone()
    sv.rope_(a, p, 0, 2, 32, 10000.0)
    sv.rope_(a, d, 0, 2, 32, 10000.0)
    sv.rope_(b, p + d, 0, 2, 32, 10000.0)
    assert torch.allclose(a, b, atol=1e-9)


def test_probe_runs_every_condition_without_leaking_slots():
    cfg, w, eng = tiny_engine()
    free0 = eng.pool.free_count()
    probes = synthetic_probes(2, 500, a_len=30, turn_len=20, b_len=25, cue_len=4, answer_len=3)
    rows = [{"probe": i, "conditions": run_probe(eng, p, CONDITIONS, tag=f"p{i}")} for i, p in enumerate(probes)]
    rep = report(rows)
    assert set(rep) == set(CONDITIONS) and all(v["n"] == 2 for v in rep.values())
    eng.radix.evict(1 << 62)  # prompts the probe prefilled stay in the prefix cache until evicted
    assert eng.pool.free_count() == free0
    eng.pool.check_invariants()


def test_route_a_conditions_and_report():
    """Route A on the tiny engine: every condition runs; without a layer subset kvcomm_sel is
    K3; on a subset engine whose subset is every layer, K2 / kvcomm_sel equal the full
    engine's K2 / K3; the report pairs conditions with bootstrap intervals."""
    from octopus_b200.baselines.route_a import CONDITIONS as RA, parse_layers, report as ra_report, run_one
    from octopus_b200.serving.engine import Engine

    cfg, w, eng = tiny_engine()
    probes = synthetic_probes(3, 500, a_len=30, turn_len=20, b_len=30, cue_len=4, answer_len=3)
    req = [7, 8, 9, 10]
    rows = [{"probe": i, "conditions": run_one(eng, None, p, RA, f"r{i}", req, 5)} for i, p in enumerate(probes)]
    c0 = rows[0]["conditions"]
    assert set(c0) == set(RA) and c0["kvcomm_sel"]["same_as"] == "K3" and c0["summary"]["summary_tokens"] == 5
    rep = ra_report(rows)
    assert rep["pairs"]["K2 - K3"]["n"] == 3 and len(rep["pairs"]["K2 - K3"]["ci95"]) == 2
    assert parse_layers("0-1", cfg.layers) == [0, 1] and parse_layers("all", cfg.layers) is None
    sub = Engine(cfg, w, kv_slots=20000, max_batch=16, device="cpu", mount_layers=[0, 1])
    r = run_one(eng, sub, probes[0], ("K2", "K3", "kvcomm_sel"), "s", req, 5)
    assert r["K2"]["layers"] == "subset" and r["kvcomm_sel"]["output"] == c0["K3"]["output"]
    assert r["K2"]["output"] == c0["K2"]["output"]
