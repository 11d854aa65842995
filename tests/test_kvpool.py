"""Native KV manager: slot refcounts, radix prefix cache, eviction fuzz (pool balance,
no double free, no freed-but-held slot)."""
import numpy as np
import pytest

from octopus_b200 import _native


def test_alloc_refcount_free_once():
    p = _native.SlotPool(100)
    s = p.alloc(10)
    assert len(s) == 10 and p.free_count() == 90
    p.incref(s[:3])
    assert p.decref(s) == 7
    assert p.decref(s[:3]) == 3
    assert p.free_count() == 100
    with pytest.raises(RuntimeError):
        p.decref(s[:1])
    assert p.check_invariants()


def test_radix_match_insert_split_evict():
    p = _native.SlotPool(1000)
    r = _native.RadixCache(p)
    toks = np.arange(1, 21, dtype=np.int32)
    sl = p.alloc(20)
    assert r.insert(0, toks, sl) == 20
    p.decref(sl)  # the request's own reference; the tree keeps its own
    n, got, h = r.match(0, np.r_[toks[:12], 99].astype(np.int32))
    assert n == 12 and list(got) == list(sl[:12])
    r.release_handle(h)
    n2, _, h2 = r.match(1, toks)  # other namespace (weight version): no hit
    assert n2 == 0
    r.release_handle(h2)
    n3, got3, h3 = r.match(0, toks)
    r.lock(h3)
    assert r.evict(1000) == 0  # locked path cannot be evicted
    r.unlock(h3)
    r.release_handle(h3)
    assert r.evict(1000) == 20
    assert p.free_count() == 1000 and p.check_invariants()


def test_zero_copy_fuzz_pool_balance():
    rng = np.random.default_rng(0)
    p = _native.SlotPool(5000)
    r = _native.RadixCache(p)
    held = []  # (slots) references held by "cursors"/"mounts"
    for step in range(400):
        op = rng.integers(0, 4)
        if op == 0:  # a request: match, allocate the rest, insert, keep as cursor
            base = rng.integers(1, 5, size=rng.integers(5, 60)).astype(np.int32)
            n, got, h = r.match(int(rng.integers(0, 2)), base)
            r.release_handle(h)
            need = len(base) - n
            new = p.alloc(need)
            if need and len(new) < need:
                r.evict(need)
                new = p.alloc(need)
                if len(new) < need:
                    continue
            slots = np.r_[np.asarray(got, np.int64), new].astype(np.int64)
            if len(got):
                p.incref(np.asarray(got, np.int64))
            r.insert(0, base, slots)
            held.append(slots)
        elif op == 1 and held:  # a mount: another holder of a random range
            s = held[rng.integers(0, len(held))]
            a = rng.integers(0, len(s))
            seg = s[a:]
            p.incref(seg)
            held.append(seg)
        elif op == 2 and held:
            s = held.pop(rng.integers(0, len(held)))
            p.decref(s)
        else:
            r.evict(int(rng.integers(1, 200)))
        assert p.check_invariants()
        for s in held:
            for x in s[:3]:
                assert p.refcount(int(x)) > 0
    for s in held:
        p.decref(s)
    r.evict(1 << 40)
    assert p.free_count() == 5000


def test_slot_runs_come_out_ascending_and_consecutive():
    """Freed slots coalesce into address-ordered runs; an allocation takes the lowest run
    that holds it whole, so a request's slots are consecutive and ascending (the decode
    kernels' tiled copies need that), and a fragmented pool still hands out ascending
    pieces of the lowest runs."""
    from octopus_b200._native import SlotPool

    p = SlotPool(64)
    a, b, c = p.alloc(8), p.alloc(8), p.alloc(8)
    assert list(a) == list(range(8)) and list(c) == list(range(16, 24))
    p.decref(np.asarray(b[::-1]))          # freed in any order: one run [8, 16)
    p.decref(np.asarray(a))                # merges into [0, 16)
    d = p.alloc(12)
    assert list(d) == list(range(12))
    e = p.alloc(10)                        # [12, 16) is too short: the run after c
    assert list(e) == list(range(24, 34))
    assert len(p.alloc(35)) == 0           # 34 free
    f = p.alloc(34)                        # no single run holds it: [12, 16), then [34, 64)
    assert list(f) == [12, 13, 14, 15] + list(range(34, 64))
    assert p.free_count() == 0 and p.check_invariants()
    for x in (c, d, e, f):
        p.decref(np.asarray(x))
    assert p.free_count() == 64 and p.check_invariants()
    assert list(p.alloc(64)) == list(range(64))
