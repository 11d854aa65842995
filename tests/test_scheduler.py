"""Continuous batching on the CPU engine: requests join and leave between decode chunks,
each stops at its own stop token, errors stay with their request, KV returns to the pool,
and every reply equals the same request generated alone (same sampling streams)."""
import numpy as np
import pytest
import torch

from octopus_b200.serving.engine import CursorNotFound, GenInput
from octopus_b200.serving.scheduler import Scheduler
from test_engine_cpu import tiny_engine


def _prompt(rng, n, vocab=512):
    return rng.integers(1, vocab, n).tolist()


def test_rows_join_and_leave_and_match_solo_runs():
    cfg, w, eng = tiny_engine(torch.float64)
    _, _, solo = tiny_engine(torch.float64)
    rng = np.random.default_rng(1)
    free0 = eng.pool.free_count()
    reqs = [GenInput(_prompt(rng, n), max_new_tokens=m, rid=100 + k, keep_cursor=False)
            for k, (n, m) in enumerate([(40, 50), (9, 7), (33, 23), (70, 3), (12, 40)])]
    sched = Scheduler(eng, chunk=4)
    try:
        futs = [sched.submit(r) for r in reqs[:3]]
        late = [sched.submit(r) for r in reqs[3:]]  # may arrive while the first three decode
        outs = [f.result(timeout=120) for f in futs + late]
    finally:
        sched.close()
    for r, o in zip(reqs, outs):
        ref = solo.generate([GenInput(r.input_ids, max_new_tokens=r.max_new_tokens, rid=r.rid, keep_cursor=False)])[0]
        assert o.output_ids == ref.output_ids
        assert np.allclose(o.output_logprobs, ref.output_logprobs, atol=1e-9)
        assert len(o.output_ids) == r.max_new_tokens
    assert sched.stats["relayouts"] >= 2
    eng.reset()
    assert eng.pool.free_count() == free0


def test_stop_tokens_end_rows_early_and_free_them():
    cfg, w, eng = tiny_engine(torch.float64)
    rng = np.random.default_rng(2)
    long = GenInput(_prompt(rng, 20), max_new_tokens=200, rid=7, keep_cursor=False)
    # a request whose every token is a stop token ends after its first sampled token
    short = GenInput(_prompt(rng, 20), max_new_tokens=200, rid=8, keep_cursor=False,
                     stop_ids=tuple(range(cfg.vocab_size)))
    free0 = eng.pool.free_count()
    sched = Scheduler(eng, chunk=4)
    try:
        f_long, f_short = sched.submit(long), sched.submit(short)
        o_short = f_short.result(timeout=60)
        assert not f_long.done()  # the short one left while the long one still decodes
        assert o_short.finish_reason == "stop" and len(o_short.output_ids) == 1
        # a mid-decode arrival is served before the long request ends
        f_mid = sched.submit(GenInput(_prompt(rng, 8), max_new_tokens=5, rid=9, keep_cursor=False))
        assert f_mid.result(timeout=60).finish_reason == "length"
        assert not f_long.done()
        assert len(f_long.result(timeout=120).output_ids) == 200
    finally:
        sched.close()
    eng.reset()
    assert eng.pool.free_count() == free0


def test_errors_fail_only_their_request():
    cfg, w, eng = tiny_engine()
    rng = np.random.default_rng(3)
    sched = Scheduler(eng, chunk=4)
    try:
        good = sched.submit(GenInput(_prompt(rng, 10), max_new_tokens=5, cursor_id="g"))
        bad = sched.submit(GenInput(_prompt(rng, 5), cursor="no-such-cursor", max_new_tokens=5))
        badm = sched.submit(GenInput(_prompt(rng, 5), mount=[("nope", 0, 3)], max_new_tokens=5))
        assert len(good.result(timeout=60).output_ids) == 5
        with pytest.raises(CursorNotFound):
            bad.result(timeout=60)
        with pytest.raises(CursorNotFound):
            badm.result(timeout=60)
        # a continuation of the kept cursor and a mount of it still work afterwards
        cont = sched.submit(GenInput(_prompt(rng, 4), cursor="g", max_new_tokens=3))
        mnt = sched.submit(GenInput(_prompt(rng, 4), mount=[("g", 0, 8)], max_new_tokens=3))
        assert len(cont.result(timeout=60).output_ids) == 3 and len(mnt.result(timeout=60).output_ids) == 3
    finally:
        sched.close()


def test_sampling_settings_run_one_at_a_time():
    cfg, w, eng = tiny_engine()
    rng = np.random.default_rng(4)
    sched = Scheduler(eng, chunk=2)
    try:
        fa = [sched.submit(GenInput(_prompt(rng, 6), max_new_tokens=6, temperature=1.0, keep_cursor=False))
              for _ in range(2)]
        fb = [sched.submit(GenInput(_prompt(rng, 6), max_new_tokens=6, temperature=0.5, keep_cursor=False))
              for _ in range(2)]
        assert all(len(f.result(timeout=60).output_ids) == 6 for f in fa + fb)
    finally:
        sched.close()
    assert sched.stats["finished"] == 4
