"""Full-shard (FSDP) actor on CPU / gloo, world_size 2, fp64: per-unit weight shards are
gathered into rotating staging slots layer by layer, gradients are reduce-scattered per
layer during the backward, the embedding and head once per step.  One step on two ranks
(each its own micro-batches, unequal counts) must equal one single-process Actor step
over all of them; the serving copy must equal the updated weights on every rank.  Both
weight sources are checked over two steps: layers gathered from the shards, and layers read
from the serving copy (re-gathered after each optimizer step)."""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from octopus_b200.models.config import get_config
from octopus_b200.rl.actor import Actor, OptimConfig, build_microbatch


def _data(seed=0, n=6):
    rng = np.random.default_rng(seed)
    V = 512
    root = rng.integers(1, V, 40)
    seqs = [np.r_[root, rng.integers(1, V, 24 + 4 * k)] for k in range(n)]
    adv = rng.normal(size=n)
    return seqs, adv


def _mb(idx, seqs, adv):
    flat = np.concatenate([seqs[i] for i in idx])
    cu = np.r_[0, np.cumsum([len(seqs[i]) for i in idx])]
    a = np.concatenate([np.full(len(seqs[i]), adv[i]) for i in idx])
    m = np.concatenate([np.r_[np.zeros(40), np.ones(len(seqs[i]) - 40)] for i in idx])
    return build_microbatch(flat, cu, None, m, a, np.zeros(len(flat)), pad_to=8)


CFG = dict(vocab_size=512, layers=3)
SPLIT = {0: [[0, 1], [2]], 1: [[3, 4, 5]]}  # rank 0: two micro-batches, rank 1: one


def _reference():
    cfg = get_config("tiny", **CFG)
    actor = Actor(cfg, "cpu", seed=5, dtype=torch.float64, ckpt=True, optim=OptimConfig(lr=1e-3))
    seqs, adv = _data()
    for _ in range(STEPS):
        st = actor.train_step([_mb(i, seqs, adv) for part in SPLIT.values() for i in part])
    return actor, float(st["grad_norm"])


STEPS = 2


def _worker(rank, world, port, q, gather):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        from octopus_b200.parallel.fsdp import FSDPActor

        cfg = get_config("tiny", **CFG)
        actor = FSDPActor(cfg, "cpu", seed=5, dtype=torch.float64, optim=OptimConfig(lr=1e-3), fused=False,
                          gather_weights=gather)
        seqs, adv = _data()
        for _ in range(STEPS):
            st = actor.train_step([_mb(i, seqs, adv) for i in SPLIT[rank]])
        q.put((rank, actor.serve16.numpy().copy(), float(st["grad_norm"])))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("gather", [False, True])
def test_fsdp_full_shard_two_ranks_matches_single_process(gather):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29400 + os.getpid() % 200 + (7 if gather else 0)
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, gather)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict((r, (w, g)) for r, w, g in (q.get(timeout=300) for _ in range(2)))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    ref, ref_gn = _reference()
    from octopus_b200.models.decoder import FlatLayout

    cfg = get_config("tiny", **CFG)
    l1, l2 = FlatLayout(cfg), FlatLayout(cfg, pad_multiple=2)
    want = ref.master.numpy()
    for r in (0, 1):
        w, gn = got[r]
        assert abs(gn - ref_gn) < 1e-9 * max(1.0, ref_gn), (gn, ref_gn)
        for s in l1.specs:
            a = want[l1.offsets[s.name]: l1.offsets[s.name] + l1.numel(s.name)]
            b = w[l2.offsets[s.name]: l2.offsets[s.name] + l2.numel(s.name)]
            assert np.allclose(a, b, atol=1e-10, rtol=1e-9), (r, s.name)
