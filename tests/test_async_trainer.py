"""Asynchronous trainer on CPU: rollouts are produced ahead, every trained rollout is at
most max_offpolicy versions stale (staler ones dropped), producer errors surface."""
import threading
import time

import pytest

from octopus_b200.rl.async_trainer import AsyncRLTrainer


class _Ro:
    def __init__(self, v):
        self.version, self.generated_tokens, self.rewards = v, 10, [1.0]


class _Engine:
    def __init__(self):
        self.version = 0

    def bump_version(self):
        self.version += 1


class _Env:
    def __init__(self, delay=0.0, fail_at=None):
        self.n, self.delay, self.fail_at = 0, delay, fail_at

    def rollout(self, eng):
        self.n += 1
        if self.fail_at is not None and self.n >= self.fail_at:
            raise ValueError("env broke")
        time.sleep(self.delay)
        return _Ro(eng.version)


class _Actor:
    version = 0


def _trainer(env, **kw):
    tr = AsyncRLTrainer(_Actor(), _Engine(), env, **kw)
    tr.train_on = lambda ro: {"loss": 0.5, "seen_version": ro.version}
    return tr


def test_bounded_staleness():
    tr = _trainer(_Env(), max_offpolicy=1, queue_size=2)
    try:
        for _ in range(6):
            st = tr.step()
            assert st["version_lag"] <= 1
        assert tr.engine.version == 6
    finally:
        tr.close()


def test_producer_error_surfaces():
    tr = _trainer(_Env(fail_at=2))
    try:
        tr.step()
        with pytest.raises(RuntimeError):
            for _ in range(5):
                tr.step()
    finally:
        tr.close()
    assert not any(t.name == "rollout-producer" and t.is_alive() for t in threading.enumerate())
