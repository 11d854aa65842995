"""Disaggregated asynchronous RL on CPU / gloo, world_size 2: rank 0 rolls out, rank 1
trains, one step apart (rollout k is generated with w_{k-1} while w_k is trained from
rollout k-1).  After three iterations the trainer's weights must equal a single-process
run of the same schedule, and the rollout rank must hold them too (the weight push)."""
import os

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from octopus_b200.envs.dag import DagConfig, MultiAgentDag
from octopus_b200.models.config import get_config
from octopus_b200.rl.actor import Actor, OptimConfig, build_microbatch

CFG = dict(vocab_size=512, layers=2)
DAG = dict(instances=2, samples=2, prefix_len=24, turn_len=6, role_len=3, seed=11)
MB = 10 ** 6
ITERS = 3


def _free_port():
    import socket

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _engine(w):
    from octopus_b200.serving.engine import Engine

    return Engine(get_config("tiny", **CFG), w, kv_slots=20000, max_batch=16, device="cpu")


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        from octopus_b200.rl.disagg import DisaggRLTrainer, make_groups, rollout_weights, split_roles

        cfg = get_config("tiny", **CFG)
        n_roll = split_roles(world)
        _, push = make_groups(world, n_roll)
        if rank < n_roll:
            w = rollout_weights(cfg, "cpu", world - n_roll, dtype=torch.float32, seed=5)
            tr = DisaggRLTrainer("rollout", n_rollout=n_roll, flat=w.flat, push_group=push, engine=_engine(w),
                                 env=MultiAgentDag(cfg.vocab_size, DagConfig(**DAG)), mb_tokens=MB)
        else:
            actor = Actor(cfg, "cpu", seed=5, dtype=torch.float32, optim=OptimConfig(lr=1e-3))
            tr = DisaggRLTrainer("train", n_rollout=n_roll, flat=actor.flat16, push_group=push, actor=actor,
                                 mb_tokens=MB)
        outs = [tr.step() for _ in range(ITERS)]
        q.put((rank, tr.flat.numpy().copy(), outs))
    finally:
        dist.destroy_process_group()


def _sequential():
    """The same schedule in one process: rollouts from a separate weight copy that receives
    the trainer's weights after each training step."""
    cfg = get_config("tiny", **CFG)
    from octopus_b200.rl.disagg import rollout_weights

    w = rollout_weights(cfg, "cpu", 1, dtype=torch.float32, seed=5)
    eng = _engine(w)
    env = MultiAgentDag(cfg.vocab_size, DagConfig(**DAG))
    actor = Actor(cfg, "cpu", seed=5, dtype=torch.float32, optim=OptimConfig(lr=1e-3))
    ros = [env.rollout(eng)]                       # iteration 0: rollout 0 (w0)
    for _ in range(1, ITERS):                       # iteration k: rollout k (w_{k-1}), train rollout k-1
        ros.append(env.rollout(eng))
        actor.train_step(ros[-2].microbatches(MB, build_microbatch))
        w.flat.copy_(actor.flat16)
        eng.bump_version()
    return actor.flat16.numpy().copy(), ros


def test_disaggregated_two_ranks_match_sequential_schedule():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict((r, (w, o)) for r, w, o in (q.get(timeout=300) for _ in range(2)))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want, ros = _sequential()
    w_roll, o_roll = got[0]
    w_train, o_train = got[1]
    assert np.allclose(w_train, want, atol=1e-6, rtol=1e-5)
    assert np.array_equal(w_roll, w_train)           # the push reached the rollout rank
    assert [o["generated_tokens"] for o in o_roll] == [r.generated_tokens for r in ros]
    assert o_train[0]["trained_tokens"] == 0           # nothing to train in iteration 0
    assert [o["trained_tokens"] for o in o_train[1:]] == [r.generated_tokens for r in ros[:-1]]
