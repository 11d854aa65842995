"""Replicated data parallelism over NCCL (the baseline multi-GPU actor).

Every rank holds a full actor replica and a rollout engine; gradients are summed with
one NCCL all-reduce of the flat fp32 gradient buffer before the fused AdamW, and the
loss denominator is the step's global loss-token count (all-reduced first), so the
update equals a single-process step over the union of the ranks' micro-batches.
Every rank issues the same collectives in the same order (one scalar all-reduce,
one buffer all-reduce per step), whatever its micro-batch count.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


class DataParallel:
    def __init__(self, actor, group=None, bucket_bytes: int = 1 << 30):
        self.actor = actor
        self.group = group
        self.bucket = bucket_bytes // 4

    def global_denominator(self, local: float) -> float:
        t = torch.tensor([float(local)], dtype=torch.float64, device=self.actor.device)
        dist.all_reduce(t, group=self.group)
        return float(t)

    def allreduce_grads(self):
        g = self.actor.grad
        n = g.numel()
        for a in range(0, n, self.bucket):
            dist.all_reduce(g[a: a + self.bucket], group=self.group)
        # gradients outside the flat buffer (hybrid models' linear layers and gate / conv
        # parameters), the same list in the same order on every rank
        for t in getattr(self.actor, "extra_grads", lambda: [])():
            dist.all_reduce(t, group=self.group)

    def attach_actor(self):
        """Wrap the actor's forward_backward / optimizer_step (no trainer needed)."""
        return self.attach(None)

    def attach(self, trainer):
        actor = self.actor
        fb = actor.forward_backward
        step = actor.optimizer_step

        def forward_backward(mbs, denom=None):
            local = float(sum(mb.pair_w.sum() for mb in mbs))
            return fb(mbs, self.global_denominator(local))

        def optimizer_step():
            self.allreduce_grads()
            return step()

        actor.forward_backward = forward_backward
        actor.optimizer_step = optimizer_step
        return trainer
