"""Training CLI with rl.disaggregate on CPU / gloo, two ranks (one rollout, one trainer):
two iterations with a step log on rank 0 that carries the trainer's numbers, a recover
checkpoint written by the trainer rank, then a resume that continues at step 3."""
import json
import os

import torch.multiprocessing as mp


def _free_port():
    import socket

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _args(tmp, steps):
    return ["--cpu", "model.preset=tiny", "rl.kind=dag", "rl.batch_size=2", "rl.n_samples=2", "rl.dag_prefix=32",
            "rl.dag_turn=8", "rl.disaggregate=true", "rollout.kv_gb=0.05", "rollout.max_batch=16",
            "actor.mb_tokens=65536", "actor.gradient_checkpointing=false", f"checkpoint.dir={tmp}",
            "checkpoint.save_every=0", f"total_steps={steps}"]


def _worker(rank, world, port, tmp, steps, q):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    from octopus_b200.rl import train

    q.put((rank, train.main(_args(tmp, steps))))


def _run(tmp, steps, port):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, tmp, steps, q)) for r in range(2)]
    for p in procs:
        p.start()
    rcs = dict(q.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert rcs == {0: 0, 1: 0}


def test_train_cli_disaggregated_runs_and_resumes(tmp_path):
    _run(str(tmp_path), 2, _free_port())
    run = tmp_path / "octopus-b200" / "run0"
    rows = [json.loads(x) for x in open(run / "steps.jsonl")]
    assert [r["step"] for r in rows] == [1, 2]
    assert rows[0]["generated_tokens"] > 0 and rows[0]["trained_tokens"] == 0
    assert rows[1]["trained_tokens"] == rows[0]["generated_tokens"]   # rollout 1 trained in iteration 2
    assert "loss" in rows[1] and (run / "recover" / "state.json").exists()
    _run(str(tmp_path), 3, _free_port())
    rows = [json.loads(x) for x in open(run / "steps.jsonl")]
    assert [r["step"] for r in rows] == [1, 2, 3]
