"""The run launcher on CPU: start a tiny trial in the background (watchdog-supervised
trainer in its own process group), see its status and step lines, stop it, and resume the
same trial; settings writes a run folder without training."""
import json
import sys
import time

from octopus_b200 import launch


def _wait(pred, timeout=240):
    t0 = time.time()
    while time.time() - t0 < timeout:
        if pred():
            return True
        time.sleep(1)
    return False


def _status(capsys, trial):
    launch.main(["status", "--trial", trial])
    return json.loads(capsys.readouterr().out.strip().splitlines()[-1])


def test_start_status_stop_resume(tmp_path, monkeypatch, capsys):
    monkeypatch.setenv("OCTOPUS_ROOT", str(tmp_path))
    train = ["--cpu", "model.preset=tiny", "rl.kind=dag", "rl.batch_size=2", "rl.n_samples=2", "rollout.kv_gb=0.05",
             "rollout.max_batch=16", "actor.mb_tokens=65536", "actor.gradient_checkpointing=false",
             "rl.dag_prefix=64", "rl.dag_turn=8", "total_steps=2", "checkpoint.recover_every=1"]
    assert launch.main(["start", "--trial", "t1", "--poll", "1", "--", *train]) == 0
    capsys.readouterr()
    assert _wait(lambda: _status(capsys, "t1")["last_step"] is not None)
    assert _wait(lambda: not _status(capsys, "t1")["running"])  # finished its two steps
    st = _status(capsys, "t1")
    assert st["last_step"]["step"] == 2 and st["live"]["MB_TOKENS"] == "262144"
    # resume: the trial folder exists, the trainer continues from its recover checkpoint
    train[-2] = "total_steps=3"
    assert launch.main(["start", "--trial", "t1", "--poll", "1", "--", *train]) == 0
    assert json.loads(capsys.readouterr().out)["resume"] is True
    assert _wait(lambda: _status(capsys, "t1")["last_step"]["step"] == 3)
    assert launch.main(["stop", "--trial", "t1"]) == 0


def test_stop_ends_the_process_group(tmp_path, monkeypatch, capsys):
    monkeypatch.setenv("OCTOPUS_ROOT", str(tmp_path))
    monkeypatch.setattr(launch, "trial_command",
                        lambda args, d: [sys.executable, "-c", "import time; time.sleep(600)"])
    assert launch.main(["start", "--trial", "sleepy"]) == 0
    capsys.readouterr()
    assert _status(capsys, "sleepy")["running"]
    assert launch.main(["stop", "--trial", "sleepy"]) == 0
    assert _wait(lambda: not _status(capsys, "sleepy")["running"], 30)


def test_settings_writes_a_run_folder(tmp_path, capsys):
    assert launch.main(["settings", str(tmp_path / "run"), "rl.kind=dag"]) == 0
    assert (tmp_path / "run" / "config.json").is_file() and (tmp_path / "run" / "episode_settings.json").is_file()
