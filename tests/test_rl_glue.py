"""Spool crash semantics, DP balance, run config, recover checkpoints, watchdog policy (CPU)."""
import json
import os
import time

import numpy as np
import pytest
import torch

from octopus_b200.models.config import get_config
from octopus_b200.rl import checkpoint, config, dp_balance, watchdog
from octopus_b200.rl.actor import Actor
from octopus_b200.rl.group import assign_threads, critical_path, group_step, leave_one_out
from octopus_b200.rl.spool import Spool


def traj(head):
    return {"versions": torch.tensor([head, head + 1]), "loss_mask": torch.tensor([1, 1]), "x": torch.ones(2)}


def test_spool_lifecycle_one_group_per_task(tmp_path):
    sp = Spool(str(tmp_path), log=lambda *a: None)
    sp.save(traj(3), "taskA")
    time.sleep(0.01)
    sp.save(traj(4), "taskA")
    sp.save(traj(4), "taskB")
    assert sp.recover(version=4) == 2
    assert sp.counts()["resume"] == 2
    t = sp.take(version=5, max_offpolicy=2, task="taskA")
    assert t and t["octopus_spool"].endswith(".pt")
    # taskA's group is out: another call of taskA while none left for it
    assert sp.take(version=5, max_offpolicy=2, task="taskC")["x"] is not None  # takes taskB's
    assert sp.take(version=5, max_offpolicy=2, task="taskA") == {}
    sp.consume([t])
    assert sp.counts()["trained"] == 1
    sp.commit()
    assert sp.counts()["trained"] == 0


def test_spool_drops_stale_groups(tmp_path):
    sp = Spool(str(tmp_path), log=lambda *a: None)
    sp.save(traj(1), "old")
    sp.recover(version=1)
    assert sp.take(version=10, max_offpolicy=2, task="x") is None
    assert sp.counts()["resume"] == 0


def test_longest_first_balance():
    w = [9, 7, 6, 5, 4, 3, 2]
    parts = dp_balance.longest_first(w, 2)
    loads = [sum(w[i] for i in p) for p in parts]
    assert abs(loads[0] - loads[1]) <= 2
    assert sorted(i for p in parts for i in p) == list(range(len(w)))


def test_config_yaml_and_overrides(tmp_path):
    p = tmp_path / "run.yaml"
    p.write_text("seed: 3\nactor:\n  lr: 1.0e-5\nrl:\n  n_samples: 8\n")
    cfg = config.load(str(p), ["actor.mb_tokens=4096", "rollout.temperature=0.7", "actor.sharded=false"])
    assert cfg.seed == 3 and cfg.actor.lr == 1e-5 and cfg.rl.n_samples == 8
    assert cfg.actor.mb_tokens == 4096 and cfg.rollout.temperature == 0.7 and cfg.actor.sharded is False
    with pytest.raises(KeyError):
        config.load(None, []) and config._apply(cfg, {"nope": 1})


def test_live_env(tmp_path, monkeypatch):
    f = tmp_path / "live.env"
    f.write_text("MB_TOKENS=65536\nACT_GPU_GB=12.5\nJUNK=1\n")
    monkeypatch.setenv("OCTOPUS_LIVE_ENV", str(f))
    assert config.live_env() == {"MB_TOKENS": 65536, "ACT_GPU_GB": 12.5}


def test_recover_checkpoint_roundtrip(tmp_path):
    cfg = get_config("tiny", layers=1, vocab_size=512)
    a = Actor(cfg, "cpu", seed=1, dtype=torch.float32)
    a.exp_avg.normal_()
    a.step_count = 7
    checkpoint.save(a, str(tmp_path), step=7, dataloader_state={"pos": 11})
    b = Actor(cfg, "cpu", seed=2, dtype=torch.float32)
    st = checkpoint.load(b, str(tmp_path))
    assert st["step"] == 7 and st["dataloader"]["pos"] == 11
    assert torch.equal(a.flat16, b.flat16) and torch.equal(a.exp_avg, b.exp_avg) and b.step_count == 7


def test_watchdog_policy(tmp_path):
    d = watchdog.decide(watchdog.Facts(False, 1, "RuntimeError: CUDA out of memory"), {})
    assert d.action == "resume" and d.mb_tokens_factor == 0.9
    d = watchdog.decide(watchdog.Facts(False, 1, "CUDA out of memory"), {"oom": 3})
    assert d.action == "stop"
    tb = 'Traceback (most recent call last):\n  File "/x/octopus_b200/rl/actor.py", line 3, in f\nValueError'
    assert watchdog.decide(watchdog.Facts(False, 1, tb), {}).action == "needs_main"
    assert watchdog.decide(watchdog.Facts(True, None, "step 3 loss nan grad_norm 1"), {}).action == "resume"
    now = time.time()
    assert watchdog.decide(watchdog.Facts(True, None, "ok", now - 9000, now), {}).action == "resume"
    assert watchdog.decide(watchdog.Facts(True, None, "ok", now - 10, now), {}).action == "continue"
    live = tmp_path / "live.env"
    assert watchdog.cut_mb_tokens(str(live), 0.9) == 235520


def test_group_credit():
    assert leave_one_out([1, 1, 1]) == [0, 0, 0]
    a = leave_one_out([1.0, -1.0, -1.0, -1.0])
    assert abs(a[0] - 2.0) < 1e-9 and abs(sum(a)) < 1e-9
    eps = [{"y": 1, "branches": [{"key": "fork0-branch-0"}]}, {"y": 0, "branches": []}]
    group_step(eps)
    assert eps[0]["A_main"] == 2.0 and eps[0]["branches"][0]["A_branch"] == 2.0
    ep = {"A_main": 1.0, "R": 1.0, "branches": [{"key": "fork0-branch-0", "A_branch": 0.5}],
          "requests": [("r1", "main", 10, 5), ("r2", "fork0/branch-0", 16, 7), ("r3", "main", 20, 3)]}
    rows = assign_threads(["r2", "r3"], ep)
    assert rows["r3"]["adv"] == 1.0 and rows["r2"]["adv"] == 0.5
    reqs = [{"thread": "main", "completion_tokens": 5}, {"thread": "fork0/branch-0", "completion_tokens": 7},
            {"thread": "fork0/branch-1", "completion_tokens": 9}, {"thread": "main", "completion_tokens": 3}]
    assert critical_path(reqs) == 17


def test_watchdog_supervise_restarts_after_oom(tmp_path):
    """A child that fails with a CUDA OOM is restarted with MB_TOKENS cut by 10% in the live
    env file (which it sees through OCTOPUS_LIVE_ENV); its second run finishes."""
    import sys

    log, live, marker = tmp_path / "run.log", tmp_path / "live.env", tmp_path / "ran_once"
    live.write_text("MB_TOKENS=100000\n")
    child = (f"import os, sys, pathlib\n"
             f"m = pathlib.Path({str(marker)!r})\n"
             f"print('live', open(os.environ['OCTOPUS_LIVE_ENV']).read().strip(), flush=True)\n"
             f"if not m.exists():\n"
             f"    m.write_text('1'); print('torch.OutOfMemoryError: CUDA out of memory', flush=True); sys.exit(1)\n"
             f"print('step 1 done', flush=True)\n")
    reports = []
    rc = watchdog.supervise([sys.executable, "-c", child], str(log), str(live), poll_s=1.0, report=reports.append)
    assert rc == 0
    assert "MB_TOKENS=89088" in live.read_text()  # 100000 * 0.9, rounded down to a multiple of 1024
    text = log.read_text()
    assert "out of memory" in text and "MB_TOKENS=89088" in text and "step 1 done" in text
    acts = [json.loads(r)["action"] for r in reports]
    assert acts == ["resume", "stop"]


def test_trainer_split_is_longest_first():
    from octopus_b200.rl.trainer import RLTrainer, TrainerConfig

    class MB:
        def __init__(self, n):
            self.n_tree, self.n_flat = n, n

    class FakeActor:
        def train_step(self, mbs):
            self.got = mbs
            return {"loss": 0.0}

    mbs = [MB(n) for n in (10, 900, 20, 800, 30)]

    class Ro:
        def microbatches(self, cap, build):
            return mbs

    shares = []
    for k in range(2):
        a = FakeActor()
        RLTrainer(a, None, None, TrainerConfig(mb_shard=(k, 2))).train_on(Ro())
        shares.append(sorted(m.n_tree for m in a.got))
    assert shares == [[900], [10, 20, 30, 800]]  # 900 | 800 + 30 + 20 + 10


def test_push_weights_after_a_step(tmp_path, monkeypatch):
    """rollout.push_hosts: each weight version is written under the run folder and handed
    to the tar-over-ssh push for every host (the push itself is faked here)."""
    from octopus_b200.rl import adapter_push, train

    calls = []
    monkeypatch.setattr(adapter_push, "push_adapter", lambda src, hosts, dest: calls.append((src, hosts, dest)) or {})
    cfg = config.load(None, ["rollout.push_hosts=h1, h2", "rollout.push_dir=/srv/w"])
    actor = Actor(get_config("tiny", layers=1), "cpu", dtype=torch.float32)
    actor.version = 3
    train._push_weights(actor, cfg, str(tmp_path))
    (src, hosts, dest), = calls
    assert hosts == ["h1", "h2"] and dest == "/srv/w/v3" and src.endswith("push/v3")
    assert any(f.endswith(".safetensors") for f in os.listdir(src))
