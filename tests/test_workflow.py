"""Workflow glue on CPU: a forked episode with a read mount, run through the engine's
cursor/mount API, becomes per-leaf training rows (single ownership, masks, spans); the
prefix-tree trainer's logprobs on the owned tokens equal the rollout's behaviour
logprobs, and a zero-variance group is filtered."""
import numpy as np
import torch

from octopus_b200.models.config import get_config
from octopus_b200.models.decoder import FlatLayout, Weights, forward_tree, init_flat
from octopus_b200.rl.actor import build_microbatch
from octopus_b200.rl.workflow import leaves_of, plan_group_rewards, rows_to_microbatches
from octopus_b200.serving.engine import Engine, GenInput


def _engine():
    cfg = get_config("tiny", vocab_size=512, layers=2)
    lay = FlatLayout(cfg)
    w = Weights(cfg, init_flat(cfg, lay, "cpu", dtype=torch.float32, seed=5, std=0.05), lay)
    eng = Engine(cfg, w, kv_slots=20000, max_batch=16, device="cpu")
    eng.record_interactions = True
    return cfg, w, eng


def _episode(eng, rng, tag, y):
    """main: 2 replies, the second forks two branches; branch b1 reads b0's reply."""
    V = eng.cfg.vocab_size
    reqs = []

    def call(thread, ids, cursor=None, mount=(), n=5):
        rid = f"{tag}-{len(reqs)}"
        o = eng.generate([GenInput(list(ids), cursor=cursor, mount=list(mount), max_new_tokens=n, cursor_id=rid)])[0]
        reqs.append({"id": rid, "thread": thread, "prompt_tokens": o.prompt_tokens + o.cached_tokens,
                     "completion_tokens": len(o.output_ids)})
        return rid

    m0 = call("main", rng.integers(1, V, 30))
    m1 = call("main", rng.integers(1, V, 6), cursor=m0)
    b0 = call("fork1/b0", rng.integers(1, V, 4), cursor=m1)
    b0b = call("fork1/b0", rng.integers(1, V, 3), cursor=b0)
    src = eng.cursors.get(b0)
    b1 = call("fork1/b1", rng.integers(1, V, 4), cursor=m1, mount=[(b0, src.length - 5, src.length - 1)])
    return {"y": y, "requests": reqs, "branches": []}, (m0, m1, b0, b0b, b1)


def test_leaves_and_ownership():
    reqs = [{"id": "a", "thread": "main"}, {"id": "b", "thread": "main"}, {"id": "c", "thread": "fork1/x"},
            {"id": "d", "thread": "fork1/y"}, {"id": "e", "thread": "fork1/x"}]
    assert leaves_of(reqs) == ["d", "e"]


def test_workflow_rows_train_on_behaviour_logprobs():
    cfg, w, eng = _engine()
    rng = np.random.default_rng(0)
    e1, ids1 = _episode(eng, rng, "e1", 1.0)
    e2, _ = _episode(eng, rng, "e2", 0.0)
    rows = plan_group_rewards([e1, e2], eng.records)
    assert e1["A_main"] == 2.0 and e2["A_main"] == -2.0
    # leaves: b0's last reply and b1 (main's replies are adopted by b0, the first branch's first leaf)
    assert [r.rid for r in rows[:2]] == [ids1[3], ids1[4]]
    r0, r1 = rows[0], rows[1]
    rec = eng.records
    # every completion of e1 is owned exactly once
    owned = r0.loss_mask.sum() + r1.loss_mask.sum()
    assert owned == sum(rec[i]["completion"] for i in ids1)
    assert r1.mounts and r1.mounts[0][1] == ids1[2]
    mbs = rows_to_microbatches([rows], eng.records, 1 << 20, lambda *a: build_microbatch(*a, pad_to=8))
    assert len(mbs) == 1
    d = mbs[0].to_device("cpu")
    lp, _ = forward_tree(w, d.batch, ckpt=False)
    # the trainer's logprobs of the owned tokens equal the rollout's behaviour logprobs
    assert torch.allclose(lp.detach().float(), d.behav.float(), atol=2e-4)
    assert np.isclose(float(d.adv.abs().max()), 2.0)


def test_zero_variance_group_filtered():
    cfg, w, eng = _engine()
    rng = np.random.default_rng(1)
    e1, _ = _episode(eng, rng, "a", 1.0)
    e2, _ = _episode(eng, rng, "b", 1.0)
    assert plan_group_rewards([e1, e2], eng.records) == []
