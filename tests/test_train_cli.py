"""Trainer entry point on CPU: two steps of the tiny DAG run from the shipped grpo.yaml with
overrides, step log, recover checkpoint, HF save, and resume from the checkpoint."""
import json
import os

from octopus_b200.rl import train


def _args(tmp, steps):
    return ["--cpu", "model.preset=tiny", "rl.kind=dag", "rl.batch_size=2", "rl.n_samples=2", "rollout.kv_gb=0.05",
            "rollout.max_batch=16", "actor.mb_tokens=65536", "actor.gradient_checkpointing=false",
            f"checkpoint.dir={tmp}", "checkpoint.save_every=2", f"total_steps={steps}"]


def test_train_cli_runs_and_resumes(tmp_path, monkeypatch):
    from octopus_b200.envs import dag

    # a small DAG shape for CPU
    orig = dag.DagConfig.__init__

    def small(self, *a, **kw):
        orig(self, *a, **kw)
        self.prefix_len, self.turn_len, self.role_len = 32, 8, 4

    monkeypatch.setattr(dag.DagConfig, "__init__", small)
    assert train.main(_args(tmp_path, 2)) == 0
    run = tmp_path / "octopus-b200" / "run0"
    rows = [json.loads(x) for x in open(run / "steps.jsonl")]
    assert [r["step"] for r in rows] == [1, 2]
    assert all({"cache_hit_rate", "requests", "kv_usage", "host_rss_gb"} <= set(r) for r in rows)
    assert rows[0]["requests"] > 0
    assert (run / "recover" / "state.json").exists() and (run / "hf-step2").exists()
    assert os.path.exists(run / "episode_settings.json")
    # resume: continues at step 3
    assert train.main(_args(tmp_path, 3)) == 0
    rows = [json.loads(x) for x in open(run / "steps.jsonl")]
    assert [r["step"] for r in rows] == [1, 2, 3]


def test_train_cli_lora(tmp_path, monkeypatch):
    from octopus_b200.envs import dag

    orig = dag.DagConfig.__init__

    def small(self, *a, **kw):
        orig(self, *a, **kw)
        self.prefix_len, self.turn_len, self.role_len = 32, 8, 4

    monkeypatch.setattr(dag.DagConfig, "__init__", small)
    args = _args(tmp_path, 1) + ["actor.lora_rank=4", "actor.ckpt_block=2", "checkpoint.recover_every=0",
                                 "checkpoint.save_every=0"]
    args = [a for a in args if a != "actor.gradient_checkpointing=false"] + ["actor.gradient_checkpointing=true"]
    assert train.main(args) == 0


def test_train_cli_swe(tmp_path, monkeypatch):
    """rl.kind=swe: plan episodes on a local task set (tiny random policy, short replies),
    graded by hidden tests, one trained step."""
    import platform
    import sys

    import pytest

    if platform.machine() != "x86_64":
        pytest.skip("x86_64 guard")
    from dataclasses import asdict

    from octopus_b200.envs.swe.taskset import TaskSpec
    from test_swe_taskset import HIDDEN, _repo

    repo = _repo(tmp_path)
    rows = tmp_path / "tasks.jsonl"
    rows.write_text("".join(json.dumps(asdict(TaskSpec(f"org__calc-{i}", repo, "HEAD", "add() subtracts; fix it.", "",
                                                       f"{sys.executable} test_hidden.py",
                                                       {"test_hidden.py": HIDDEN}))) + "\n" for i in range(2)))
    monkeypatch.setenv("OCTOPUS_MAX_TOKENS", "6")
    monkeypatch.setenv("OCTOPUS_MAIN_MAX_CALLS", "2")
    args = [a for a in _args(tmp_path, 1) if a != "rl.kind=dag"] + [
        "rl.kind=swe", f"rl.swe_tasks={rows}", "rl.filter_zero_variance=false", "rl.swe_timeout=30",
        "checkpoint.recover_every=0", "checkpoint.save_every=0"]
    assert train.main(args) == 0
    run = tmp_path / "octopus-b200" / "run0"
    (row,) = [json.loads(x) for x in open(run / "steps.jsonl")]
    assert row["step"] == 1
