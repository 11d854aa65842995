"""Asynchronous RL: rollouts of the next steps are produced while the current step trains,
with bounded staleness (the decoupled-PPO objective corrects for the behaviour policy).

A producer thread runs `env.rollout(engine)` back to back into a queue of at most
`queue_size` finished rollouts, tagging each with the engine's weight version when it
started.  `step()` takes the next rollout whose version lag behind the actor is at most
`max_offpolicy` (staler ones are dropped and counted), trains on it, and syncs the
weights (bumping the engine version, which the producer reads before its next rollout).

With a colocated engine on the same GPU both threads issue work on that GPU; the
producer's kernels and the trainer's are ordered by the device's streams, so a weight
update never lands inside a running kernel, only between requests (as a remote
rollout server receives updates between requests).

Reference parity (behaviour): `octopus/rl/grpo.yaml` `max_head_offpolicyness: 2` with
AReaL's asynchronous rollout workers, `octopus/rl/spool.py` (head_version of a group).
"""
from __future__ import annotations

import queue
import threading
import time

from .trainer import RLTrainer


class AsyncRLTrainer(RLTrainer):
    def __init__(self, actor, engine, env, cfg=None, sync_fn=None, max_offpolicy: int = 2, queue_size: int = 1):
        super().__init__(actor, engine, env, cfg, sync_fn)
        self.max_offpolicy = max_offpolicy
        self.q: queue.Queue = queue.Queue(maxsize=queue_size)
        self._stop = threading.Event()
        self._thread = None
        self._error = None
        self.dropped = 0

    def _produce(self):
        try:
            while not self._stop.is_set():
                version = getattr(self.engine, "version", 0)
                t0 = time.perf_counter()
                ro = self.env.rollout(self.engine)
                item = (version, ro, time.perf_counter() - t0)
                while not self._stop.is_set():
                    try:
                        self.q.put(item, timeout=0.1)
                        break
                    except queue.Full:
                        continue
        except Exception as e:  # surfaced by the next step()
            self._error = e

    def start(self):
        if self._thread is None:
            self._thread = threading.Thread(target=self._produce, name="rollout-producer", daemon=True)
            self._thread.start()
        return self

    def step(self) -> dict:
        self.start()
        while True:
            if self._error is not None:
                raise RuntimeError("rollout producer failed") from self._error
            try:
                version, ro, roll_s = self.q.get(timeout=0.5)
            except queue.Empty:
                continue
            lag = getattr(self.engine, "version", 0) - version
            if lag <= self.max_offpolicy:
                break
            self.dropped += 1
        t1 = time.perf_counter()
        stats = self.train_on(ro)
        t2 = time.perf_counter()
        self.sync()
        loss = float(stats["loss"]) if not hasattr(stats["loss"], "item") else float(stats["loss"].item())
        self.steps += 1
        out = {k: (float(v) if hasattr(v, "item") else v) for k, v in stats.items()}
        out.update(loss=loss, generated_tokens=ro.generated_tokens, rollout_s=roll_s, train_s=t2 - t1,
                   sync_s=time.perf_counter() - t2, version_lag=lag, dropped=self.dropped,
                   mean_reward=sum(ro.rewards) / max(1, len(ro.rewards)))
        return out

    def close(self):
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=30)
            self._thread = None
