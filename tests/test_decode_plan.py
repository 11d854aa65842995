"""Shared-prefix decode planner (CPU): every row's keys are covered exactly once by its
segments in order, shared segments serve rows whose contexts agree, and the slot
bookkeeping fits the tables."""
import numpy as np
import pytest

from octopus_b200.ops.decode import SharedDecode


def dag_rows(n_inst=3, per=8, pre=300, plan=100, own=40, rng=None):
    rows, ctx, nxt = [], [], 0

    def take(n):
        nonlocal nxt
        r = np.arange(nxt, nxt + n)
        nxt += n
        return r

    for _ in range(n_inst):
        p = take(pre)
        for _ in range(per // 2):
            pl = take(plan)
            for _ in range(2):
                rows.append(np.concatenate([p, pl, take(own)]))
                ctx.append(pre + plan)
    return rows, np.asarray(ctx)


@pytest.mark.parametrize("use_tc", [False, True])
def test_plan_covers_every_row_once(use_tc):
    rows, ctx = dag_rows()
    starts = np.cumsum([0] + [len(r) for r in rows[:-1]])
    final = np.asarray([len(r) for r in rows])
    sd = SharedDecode(28, 4, 128, 32, device="cpu", chunk=64, min_shared=32, use_tc=use_tc)
    assert sd.plan(rows, starts, ctx, final, 32)
    S = sd.stats["segments"]
    seg_rows = sd.t_rows.view(-1, SharedDecode.SEG_STRIDE)[:S].numpy()
    st, ln, off = sd.t_start[:S].numpy(), sd.t_len[:S].numpy(), sd.t_off[:S].numpy()
    flat = np.concatenate(rows)
    for b in range(len(rows)):
        got = []
        for s in range(S):
            if b in seg_rows[s]:
                n = ln[s] if ln[s] >= 0 else final[b] - off[s]
                got.append((off[s], flat[st[s]:st[s] + n]))
        got.sort(key=lambda x: x[0])
        keys = np.concatenate([g[1] for g in got])
        assert np.array_equal(keys, rows[b]), b
    # 3 instances x 8 rows: the prefix is one segment per instance on the tcgen05 kernel (up to
    # 128 / 7 rows per tile) and two of <= 4 rows on the mma.sync kernel; planner pairs; own remainders
    per_prefix = 1 if use_tc else 2
    assert sd.stats["shared_segments"] == 3 * per_prefix + 12
    assert sd.stats["segments"] == 3 * per_prefix + 12 + 24
    assert int(sd.t_nslot[:24].max()) == sd.stats["max_slots"]


def test_plan_without_sharing_is_one_segment_per_row():
    rng = np.random.default_rng(0)
    rows = [rng.permutation(10000)[:n] for n in (50, 70, 90)]
    sd = SharedDecode(8, 8, 128, 8, device="cpu")
    assert sd.plan(rows, np.asarray([0, 50, 120]), np.asarray([40, 60, 80]), np.asarray([50, 70, 90]), 8)
    assert sd.stats["segments"] == 3 and sd.stats["shared_segments"] == 0
