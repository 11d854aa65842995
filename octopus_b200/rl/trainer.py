"""RL trainer: rollout (engine) -> prefix-tree train (actor) -> weight sync, one step.

`RLTrainer.step()` is the public end-to-end API of one RL step on one model replica:

1. rollout of the environment's episodes through the engine (cursors, mounts);
2. group credit (leave-one-out advantages, single ownership) and micro-batch packing
   of whole mount units into prefix trees under a token cap;
3. forward/backward of every micro-batch and one fused AdamW step;
4. weight sync: when the engine is colocated it reads the trainer's bf16 compute
   buffer directly (the AdamW kernel writes it in place), so the sync is a version
   bump that invalidates cached prefixes of the old weights; a separate engine copy
   (other layout or device) is refreshed by `sync_fn`.

Returns per-step stats including generated/trained tokens and phase wall times.
Reference parity: the PPOTrainer loop driven by `octopus/rl/train.py:55-137`
(rollout -> compute advantages -> ppo_update -> weight update -> recover checkpoint).
"""
from __future__ import annotations

import time
from dataclasses import dataclass

import torch

from ..utils.iostats import d2h
from .actor import Actor, build_microbatch
from .dp_balance import longest_first


@dataclass
class TrainerConfig:
    mb_tokens: int = 32768      # prefix-tree tokens per micro-batch (flat estimate)
    sync_every: int = 1
    # (index, count): this rank's share of the micro-batches when `count` ranks hold the same
    # rollout (the ranks of one tensor-parallel rollout group split its training): the
    # micro-batches are assigned largest-first by prefix-tree tokens (rl.dp_balance).
    mb_shard: tuple = (0, 1)


class RLTrainer:
    def __init__(self, actor: Actor, engine, env, cfg: TrainerConfig | None = None, sync_fn=None):
        self.actor, self.engine, self.env = actor, engine, env
        self.cfg = cfg or TrainerConfig()
        self.sync_fn = sync_fn
        self.steps = 0

    def rollout(self):
        return self.env.rollout(self.engine)

    def train_on(self, ro) -> dict:
        mbs = ro.microbatches(self.cfg.mb_tokens, build_microbatch)
        k, n = self.cfg.mb_shard
        if n > 1:  # this rank's share: micro-batches assigned longest-first by tree tokens
            mbs = [mbs[i] for i in sorted(longest_first([mb.n_tree for mb in mbs], n)[k])]
        stats = self.actor.train_step(mbs)
        stats["micro_batches"] = len(mbs)
        stats["tree_tokens"] = sum(mb.n_tree for mb in mbs)
        stats["flat_tokens"] = sum(mb.n_flat for mb in mbs)
        return stats

    def sync(self):
        if self.sync_fn is not None:
            self.sync_fn()
        self.engine.bump_version()

    def step(self) -> dict:
        t0 = time.perf_counter()
        ro = self.rollout()
        t1 = time.perf_counter()
        stats = self.train_on(ro)
        t2 = time.perf_counter()
        self.sync()
        # the step's result read back to the host (loss)
        loss = float(d2h(stats["loss"].reshape(1))[0]) if torch.is_tensor(stats["loss"]) else float(stats["loss"])
        t3 = time.perf_counter()
        self.steps += 1
        out = {k: (float(v) if torch.is_tensor(v) else v) for k, v in stats.items()}
        out.update(loss=loss, generated_tokens=ro.generated_tokens, rollout_s=t1 - t0, train_s=t2 - t1,
                   sync_s=t3 - t2, step_s=t3 - t0, mean_reward=sum(ro.rewards) / max(1, len(ro.rewards)))
        return out
