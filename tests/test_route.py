"""Session router admission (fake loads, fake clock)."""
import asyncio

import pytest

from octopus_b200.serving.route import Ended, Router


class Clock:
    def __init__(self):
        self.t = 0.0

    def __call__(self):
        return self.t


def test_sticky_sessions_and_least_inflight():
    r = Router(["a", "b"])
    s1 = r.admit("ep1")
    r.inflight[s1] += 5
    s2 = r.admit("ep2")
    assert s2 != s1
    assert r.admit("ep1") == s1  # sticky


def test_cap_blocks_new_sessions_only():
    r = Router(["a"], cap=1)
    s = r.admit("ep1")
    r.inflight[s] = 1
    assert r.admit("ep2") is None
    assert r.admit("ep1") == "a"  # admitted session never waits


def test_kv_target_and_poll_rules():
    loads = {"a": (0.95, 0, 1000), "b": (0.2, 0, 1000)}
    r = Router(["a", "b"], kv=0.9, load_fn=lambda s: loads[s])
    r.poll()
    assert r.admit("x") == "b"
    assert r.admit("y") is None  # b took a session since its last poll
    r.poll()
    assert r.admit("y") == "b"
    loads["b"] = (0.1, 3, 1000)  # queued requests close it
    r.poll()
    assert r.admit("z") is None
    assert r.admit("z", late=True) in ("a", "b")


def test_tree_budget_slots():
    loads = {"a": (0.0, 0, 1000)}
    r = Router(["a"], kv=0.5, tree_tokens=250, load_fn=lambda s: loads[s])  # 2 slots
    for k in ("t1", "t2"):
        r.poll()
        assert r.admit(k) == "a"
    r.poll()
    assert r.admit("t3") is None
    r.end("t1")
    r.poll()
    assert r.admit("t3") == "a"


def test_ended_session_refused_until_started():
    r = Router(["a"])
    r.admit("e")
    r.end("e")
    with pytest.raises(Ended):
        r.admit("e")
    r.start("e")
    assert r.admit("e") == "a"


def test_shared_dir_counts_other_routers(tmp_path):
    loads = {"a": (0.0, 0, 1000)}
    r1 = Router(["a"], kv=0.5, tree_tokens=250, shared_dir=str(tmp_path), load_fn=lambda s: loads[s])
    r2 = Router(["a"], kv=0.5, tree_tokens=250, shared_dir=str(tmp_path), load_fn=lambda s: loads[s])
    r1.poll()
    r1.admit("p")
    r1.poll()
    r1.admit("q")
    r2.poll()
    assert r2.trees("a") == 2 and r2.admit("z") is None


def test_enter_leave_async():
    async def go():
        r = Router(["a", "b"])
        s = await r.enter("k")
        await r.leave(s)
        return s

    assert asyncio.run(go()) in ("a", "b")
