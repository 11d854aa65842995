"""Continuous-batching scheduler of the rollout engine.

Requests join and leave the decode batch between decode chunks instead of waiting for a
whole static batch:

* ``submit(GenInput)`` queues a request and returns a future.
* The scheduler thread loops: admit waiting requests (one prefill for all of them, as
  many as free batch rows allow), lay out the live rows, run a decode chunk of a few
  steps (CUDA-graph replays of the engine's decode step), read the chunk's tokens back,
  and close every row that produced a stop token or reached its max_new_tokens; its
  future gets its GenOutput and its batch row is free for the next arrival.
* One sampling setting (temperature, top-p, top-k) runs at a time: a request with a
  different setting waits until the live rows of the current one have drained.
* Errors are per request: an unknown cursor, a bad mount or an allocation that fails
  even after eviction fails that request's future only.  A request that does not fit in
  the KV pool while other rows are live waits for them to finish and is then retried.

Decode chunks are short (CHUNK steps), so a request that stops early holds its row for at
most CHUNK - 1 wasted steps, and an arrival waits at most one chunk before its prefill.
Sampling streams are per request (rid, position), so a reply does not depend on which
other requests shared its batch.

Reference parity (behaviour): the SGLang scheduler the reference serves through
(continuous batching, per-request stop, prefill-only requests: `octopus/serving/
kv_mount.py:565-569`), with the cursor / mount request semantics of the engine.
"""
from __future__ import annotations

import collections
import concurrent.futures as cf
import threading

from .engine import Engine, GenInput, GenOutput, OutOfKV

CHUNK = 16


def sampling_key(inp: GenInput) -> tuple:
    return float(inp.temperature), float(inp.top_p), int(inp.top_k)


class Scheduler:
    def __init__(self, engine: Engine, chunk: int = CHUNK, max_rows: int | None = None):
        if not engine.supports_continuous:
            raise ValueError("this engine runs static batches only (Engine.generate)")
        self.engine = engine
        self.chunk = int(chunk)
        self.max_rows = min(max_rows or engine.max_batch, engine.max_batch)
        self._waiting: collections.deque = collections.deque()  # (GenInput, Future)
        self._cv = threading.Condition()
        self._live: list = []  # (request, future), in decode-row order
        self._key = None
        self._stop = False
        self.stats = {"admitted": 0, "finished": 0, "failed": 0, "chunks": 0, "relayouts": 0}
        self._thread = threading.Thread(target=self._loop, name="octopus-scheduler", daemon=True)
        self._thread.start()

    # ------------------------------------------------------------------ API
    def submit(self, inp: GenInput) -> cf.Future:
        fut: cf.Future = cf.Future()
        with self._cv:
            if self._stop:
                raise RuntimeError("scheduler closed")
            self._waiting.append((inp, fut))
            self._cv.notify()
        return fut

    def generate(self, inputs: list[GenInput]) -> list[GenOutput]:
        """Blocking convenience: submit all, wait for all (raises the first failure)."""
        futs = [self.submit(i) for i in inputs]
        return [f.result() for f in futs]

    @property
    def pending(self) -> int:
        return len(self._waiting)

    @property
    def running(self) -> int:
        return len(self._live)

    def close(self, timeout: float = 30.0):
        with self._cv:
            self._stop = True
            self._cv.notify()
        self._thread.join(timeout)

    # ------------------------------------------------------------------ loop pieces
    def _take_admissible(self) -> list:
        """Waiting requests of the running sampling setting (or of the oldest waiting one
        when nothing is live), up to the free rows.  Called with the lock held."""
        free = self.max_rows - len(self._live)
        if free <= 0 or not self._waiting:
            return []
        key = self._key if self._live else sampling_key(self._waiting[0][0])
        picked, keep = [], collections.deque()
        while self._waiting:
            inp, fut = self._waiting.popleft()
            if fut.cancelled():
                continue
            if len(picked) < free and sampling_key(inp) == key:
                picked.append((inp, fut))
            else:
                keep.append((inp, fut))
        self._waiting = keep
        if picked:
            self._key = key
        return picked

    def _admit(self, batch: list) -> bool:
        """Prefill `batch`; returns whether the live set changed."""
        results = self.engine.admit([inp for inp, _ in batch])
        changed, retry = False, []
        for (inp, fut), res in zip(batch, results):
            if isinstance(res, OutOfKV) and self._live:
                retry.append((inp, fut))  # room frees up when live rows finish
                continue
            if isinstance(res, Exception):
                self.stats["failed"] += 1
                fut.set_exception(res)
                continue
            self.stats["admitted"] += 1
            if self._done(res):
                self._close(res, fut)
            else:
                self._live.append((res, fut))
                changed = True
        if retry:
            with self._cv:
                self._waiting.extendleft(reversed(retry))
        return changed

    @staticmethod
    def _done(r) -> bool:
        inp = r.inp
        if inp.prefill_only or len(r.out_tok) >= inp.max_new_tokens:
            return True
        return bool(inp.stop_ids) and any(t in inp.stop_ids for t in r.out_tok)

    def _close(self, r, fut):
        try:
            out = self.engine.finish(r)
        except Exception as e:  # noqa: BLE001
            self.stats["failed"] += 1
            fut.set_exception(e)
            return
        self.stats["finished"] += 1
        fut.set_result(out)

    def _drain(self):
        for _, fut in list(self._waiting) + self._live:
            if not fut.done():
                fut.set_exception(RuntimeError("scheduler closed"))
        for r, _ in self._live:
            self.engine._abandon(r)
        self._waiting.clear()
        self._live.clear()

    def _loop(self):
        eng = self.engine
        dirty, B = True, 0
        while True:
            with self._cv:
                while not self._stop and not self._waiting and not self._live:
                    self._cv.wait()
                if self._stop:
                    self._drain()
                    return
                batch = self._take_admissible()
            try:
                if batch and self._admit(batch):
                    dirty = True
                if not self._live:
                    continue
                rows = [r for r, _ in self._live]
                steps = max(1, min(self.chunk, max(r.inp.max_new_tokens - len(r.out_tok) for r in rows)))
                if dirty:
                    B = eng.layout_rows(rows, self.chunk)
                    self.stats["relayouts"] += 1
                    dirty = False
                toks, lps = eng.decode_chunk(len(rows), B, steps, self._key[0])
                self.stats["chunks"] += 1
                still = []
                for k, (r, fut) in enumerate(self._live):
                    r.out_tok.extend(int(x) for x in toks[k])
                    r.out_lp.extend(float(x) for x in lps[k])
                    if self._done(r):
                        self._close(r, fut)
                        dirty = True
                    else:
                        still.append((r, fut))
                self._live = still
            except Exception as e:  # noqa: BLE001  (an engine failure fails the live rows; the loop goes on)
                for r, fut in self._live:
                    eng._abandon(r)
                    if not fut.done():
                        fut.set_exception(e)
                self.stats["failed"] += len(self._live)
                self._live = []
                dirty = True
