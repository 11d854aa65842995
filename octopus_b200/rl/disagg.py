"""Disaggregated asynchronous RL: rollout and training on disjoint GPU sets, one step apart.

Ranks [0, R) each run a rollout engine replica over their share of the environment;
ranks [R, N) hold the actor, sharded over the trainer group.  Iteration k:

    rollout ranks   generate rollout k with weights w_{k-1}
    trainer ranks   train on rollout k-1, producing w_k            (at the same time)
    exchange        rollout k moves rollout rank i -> trainer rank R + i % T (a pickled
                    object over the process group), and w_k (the full bf16 buffer) is
                    broadcast from the first trainer rank to every rollout rank

so every rollout is trained exactly once, by an actor one weight version ahead of the
policy that sampled it; the decoupled-PPO objective (behaviour log-probs recorded at
sampling) corrects for that lag.  The iteration takes max(rollout, train) + exchange
instead of rollout + train: rollout is bound by streaming the weights once per decode
step on every replica, so halving the replicas costs it less than doubling the trainer's
share saves.

Reference parity (behaviour): the reference trains asynchronously with bounded staleness
(`octopus/rl/grpo.yaml` `max_head_offpolicyness: 2`, AReaL rollout workers on their own
GPUs, weights pushed to the rollout servers after each step).
"""
from __future__ import annotations

import time

import torch
import torch.distributed as dist

from ..utils.iostats import d2h
from .actor import build_microbatch


class DisaggRLTrainer:
    """One rank's side of the disaggregated loop.

    role "rollout": `engine` (its weights are `flat`, the engine's bf16 buffer) and `env`;
    role "train": `actor` (its full bf16 serving buffer is `flat`: `flat16` / `serve16`).
    `n_rollout` ranks [0, n_rollout) roll out, the others train; `push_group` holds the
    first trainer rank and every rollout rank (the weight broadcast)."""

    def __init__(self, role: str, *, n_rollout: int, flat: torch.Tensor, push_group, engine=None, env=None,
                 actor=None, mb_tokens: int = 32768, report: bool = False):
        assert role in ("rollout", "train")
        self.role = role
        self.rank, self.world = dist.get_rank(), dist.get_world_size()
        self.n_rollout = n_rollout
        self.n_train = self.world - n_rollout
        assert self.n_train >= 1 and n_rollout >= 1
        self.flat, self.push_group = flat, push_group
        self.engine, self.env, self.actor = engine, env, actor
        self.mb_tokens = mb_tokens
        self.report = report
        self.pending = []    # trainer: rollouts received, not trained yet
        self.steps = 0
        self.version = 0     # weight version this rank holds
        if self.role == "rollout" or self.rank == n_rollout:  # the pushed buffer has one size on both sides
            n = torch.tensor([flat.numel()], dtype=torch.int64, device=flat.device)
            dist.broadcast(n, src=n_rollout, group=push_group)
            if int(n.item()) != flat.numel():
                raise ValueError(f"weight buffer of {flat.numel()} elements, the trainer's has {int(n.item())}: "
                                 "build the rollout weights with rollout_weights()")

    # ------------------------------------------------------------------ exchange
    def _sources(self):
        """Rollout ranks whose rollouts this trainer rank trains."""
        j = self.rank - self.n_rollout
        return [i for i in range(self.n_rollout) if i % self.n_train == j]

    def _exchange(self, ro):
        """Rollouts -> trainer ranks, then weights -> rollout ranks (every rank calls this)."""
        if self.role == "rollout":
            dist.send_object_list([ro], dst=self.n_rollout + self.rank % self.n_train)
        else:
            for src in self._sources():
                box = [None]
                dist.recv_object_list(box, src=src)
                self.pending.append(box[0])
        self.push_weights()
        self.version = self.steps

    def push_weights(self):
        """The first trainer rank's bf16 weights -> every rollout rank (each of these ranks calls it)."""
        if self.role == "rollout" or self.rank == self.n_rollout:
            dist.broadcast(self.flat, src=self.n_rollout, group=self.push_group)
        if self.role == "rollout":
            self.engine.bump_version()  # cached prefixes of the old weights are not reused

    # ------------------------------------------------------------------ one iteration
    def step(self) -> dict:
        t0 = time.perf_counter()
        out = {"role": self.role, "generated_tokens": 0, "trained_tokens": 0}
        ro = None
        if self.role == "rollout":
            ro = self.env.rollout(self.engine)
            out["generated_tokens"] = ro.generated_tokens
            out["mean_reward"] = sum(ro.rewards) / max(1, len(ro.rewards))
            t1 = time.perf_counter()
            out["rollout_s"] = t1 - t0
        else:
            batches, self.pending = self.pending, []
            mbs = [mb for r in batches for mb in r.microbatches(self.mb_tokens, build_microbatch)]
            if self.steps > 0:  # (iteration 0 has nothing to train yet, on every trainer rank alike)
                stats = self.actor.train_step(mbs)
                loss = stats["loss"]
                out["loss"] = float(d2h(loss.reshape(1))[0]) if torch.is_tensor(loss) else float(loss)
                out["trained_tokens"] = int(sum(float(mb.pair_w.sum()) for mb in mbs))
                out["tree_tokens"] = int(sum(mb.n_tree for mb in mbs))
                out["flat_tokens"] = int(sum(mb.n_flat for mb in mbs))
                out["micro_batches"] = len(mbs)
            t1 = time.perf_counter()
            out["train_s"] = t1 - t0
        self._exchange(ro)
        self.steps += 1
        t2 = time.perf_counter()
        out.update(sync_s=t2 - t1, step_s=t2 - t0, version=self.version)
        if self.report:  # the first trainer rank's numbers travel to rank 0 (the run's log)
            if self.rank == self.n_rollout:
                dist.send_object_list([out], dst=0)
            elif self.rank == 0:
                box = [None]
                dist.recv_object_list(box, src=self.n_rollout)
                own = ("trained_tokens", "loss", "tree_tokens", "flat_tokens", "micro_batches", "train_s")
                out.update({k if k in own else f"train_{k}": v for k, v in box[0].items()
                            if k not in ("role", "generated_tokens")})
        return out


def split_roles(world: int, n_rollout: int = 0) -> int:
    """Rollout ranks of a disaggregated job: half of the GPUs by default (the larger half
    for odd counts, so every trainer rank has a rollout rank to train on)."""
    if world < 2:
        raise ValueError("disaggregated RL needs at least two ranks")
    r = n_rollout or (world + 1) // 2
    if not world - r <= r:
        raise ValueError(f"{r} rollout ranks cannot feed {world - r} trainer ranks")
    return max(1, min(world - 1, r))


def rollout_weights(cfg, device, n_train: int, dtype=torch.bfloat16, seed: int = 0):
    """A rollout rank's weights: the flat layout of an actor sharded over `n_train` ranks
    (same padding, so the trainer's buffer broadcasts into it as is), random-init like the
    actor's (same seed)."""
    from ..models.decoder import FlatLayout, Weights, init_flat

    layout = FlatLayout(cfg, pad_multiple=n_train)
    flat = init_flat(cfg, layout, device, dtype=dtype, seed=seed)
    return Weights(cfg, flat, layout)


def make_groups(world: int, n_rollout: int):
    """(trainer group, push group); every rank creates both, in the same order."""
    train_group = dist.new_group(list(range(n_rollout, world)))
    push_group = dist.new_group([n_rollout] + list(range(n_rollout)))
    return train_group, push_group
