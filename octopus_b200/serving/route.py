"""Session router: which rollout server a request goes to.

One session is one episode tree; every thread of it stays on one server (cursors,
mounts and prefix reuse are per server).  A new session is placed on the server with
the fewest of this router's requests in flight; with a cap (> 0) it waits until some
server has fewer than `cap` in flight (follow-up requests of admitted sessions never
wait).  With a KV target (kv > 0) a poller reads every server's ``/v1/loads`` and a new
session only goes to a server below the target with nothing queued that took no new
session since its last poll; with a tree budget (tree_tokens > 0) a server takes a new
tree only while it holds fewer than max(1, kv * max_tokens / tree_tokens) trees (the
counts of other routers on the host are read from per-router files in a shared
directory).  After `wait` seconds a waiting session takes a server under the cap
anyway.  Sessions expire after EXPIRE seconds without a request; an ended session is
never admitted again until it is started again.  Among open servers one is drawn at
random in proportion to its free slots (or free KV below the target).

Reference parity (behaviour): `octopus/serving/route.py:103-299` (Router.enter, _poll,
server_load, end/start, shared tree counts).
"""
from __future__ import annotations

import asyncio
import json
import os
import random
import time
import urllib.request
import uuid
from collections import OrderedDict

POLL = 2.0
STALE = 60.0
EXPIRE = 3600.0
ENDED_KEPT = 4096


def server_load(addr: str, timeout: float = POLL):
    """(token_usage, waiting requests, max tokens) of a server's /v1/loads; None if unreadable."""
    try:
        with urllib.request.urlopen(f"http://{addr}/v1/loads", timeout=timeout) as r:
            d = json.load(r)
        loads = d.get("loads") or [d]
        return (max(float(x.get("token_usage", 0.0)) for x in loads),
                sum(int(x.get("num_waiting_reqs", 0)) for x in loads),
                sum(int(x.get("max_total_num_tokens", x.get("kv_slots", 0)) or 0) for x in loads))
    except Exception:
        return None


class Ended(RuntimeError):
    """The session ended while its first request waited for admission."""


class Router:
    def __init__(self, servers: list[str], cap: int = 0, kv: float = 0.0, wait: float = 300.0, tree_tokens: int = 0,
                 shared_dir: str | None = None, load_fn=server_load, clock=time.monotonic, rng=None):
        self.servers = list(servers)
        self.cap, self.kv, self.wait, self.tree_tokens = cap, kv, wait, tree_tokens
        self.inflight = dict.fromkeys(self.servers, 0)
        self.session: dict[str, str] = {}
        self.seen: dict[str, float] = {}
        self.ended: OrderedDict[str, None] = OrderedDict()
        self.loads: dict[str, tuple | None] = dict.fromkeys(self.servers, None)
        self.took_since_poll: set[str] = set()
        self.load_fn, self.clock = load_fn, clock
        self.rng = rng or random.Random(0)
        self.shared_dir = shared_dir
        self.id = uuid.uuid4().hex[:8]
        self._cond: asyncio.Condition | None = None
        self.admitted_late = 0

    # ------------------------------------------------------------------ bookkeeping
    def trees(self, server: str) -> int:
        own = sum(1 for s in self.session.values() if s == server)
        return own + self._others(server)

    def _others(self, server: str) -> int:
        if not self.shared_dir or not os.path.isdir(self.shared_dir):
            return 0
        n, now = 0, time.time()
        for fn in os.listdir(self.shared_dir):
            if fn == f"{self.id}.json":
                continue
            p = os.path.join(self.shared_dir, fn)
            try:
                if now - os.path.getmtime(p) > STALE:
                    continue
                n += int(json.load(open(p)).get(server, 0))
            except (OSError, ValueError):
                continue
        return n

    def _publish(self):
        if not self.shared_dir:
            return
        os.makedirs(self.shared_dir, mode=0o700, exist_ok=True)
        counts = {s: sum(1 for v in self.session.values() if v == s) for s in self.servers}
        tmp = os.path.join(self.shared_dir, f".{self.id}.tmp")
        with open(tmp, "w") as f:
            json.dump(counts, f)
        os.replace(tmp, os.path.join(self.shared_dir, f"{self.id}.json"))

    def slots(self, server: str) -> int | None:
        ld = self.loads.get(server)
        if not (self.kv > 0 and self.tree_tokens > 0 and ld):
            return None
        return max(1, int(self.kv * ld[2] / self.tree_tokens))

    def poll(self):
        for s in self.servers:
            self.loads[s] = self.load_fn(s)
        self.took_since_poll.clear()
        now = self.clock()
        for k, t in list(self.seen.items()):
            if now - t > EXPIRE:
                self._drop(k)
        self._publish()

    def _drop(self, key):
        self.session.pop(key, None)
        self.seen.pop(key, None)

    def end(self, key: str):
        self._drop(key)
        self.ended[key] = None
        while len(self.ended) > ENDED_KEPT:
            self.ended.popitem(last=False)
        self._publish()

    def start(self, key: str):
        self.ended.pop(key, None)

    # ------------------------------------------------------------------ placement
    def _open(self, s: str) -> bool:
        if self.cap and self.inflight[s] >= self.cap:
            return False
        if self.kv <= 0:
            return True
        ld = self.loads.get(s)
        if ld is None:  # unreadable: open, one new session per poll
            return s not in self.took_since_poll
        usage, waiting, _ = ld
        if usage >= self.kv or waiting > 0 or s in self.took_since_poll:
            return False
        sl = self.slots(s)
        return sl is None or self.trees(s) < sl

    def choose(self, late: bool = False) -> str | None:
        if late:
            cands = [s for s in self.servers if not self.cap or self.inflight[s] < self.cap]
            if not cands:
                return None
            return min(cands, key=lambda s: ((self.loads.get(s) or (1.0,))[0], self.inflight[s]))
        cands = [s for s in self.servers if self._open(s)]
        if not cands:
            return None
        if self.kv <= 0:
            low = min(self.inflight[s] for s in cands)
            return self.rng.choice([s for s in cands if self.inflight[s] == low])
        readable = [s for s in cands if self.loads.get(s) is not None]
        if not readable:
            return min(cands, key=lambda s: self.inflight[s])

        def weight(s):
            sl = self.slots(s)
            if sl is not None:
                return max(sl - self.trees(s), 1e-6)
            usage, _, mx = self.loads[s]
            return max(mx * (self.kv - usage), 1e-6)

        w = [weight(s) for s in readable]
        return self.rng.choices(readable, weights=w)[0]

    def admit(self, key: str, late: bool = False) -> str | None:
        """Synchronous placement (None: nothing open now)."""
        if key in self.ended:
            raise Ended(key)
        if key in self.session:
            return self.session[key]
        s = self.choose(late)
        if s is not None:
            self.session[key] = s
            self.took_since_poll.add(s)
            if late:
                self.admitted_late += 1
            self._publish()
        return s

    async def enter(self, key: str) -> str:
        """Server for a request of session `key`, waiting for admission if needed; pair with leave()."""
        if self._cond is None:
            self._cond = asyncio.Condition()
        t0 = self.clock()
        while True:
            s = self.admit(key, late=self.clock() - t0 >= self.wait)
            if s is not None:
                self.inflight[s] += 1
                self.seen[key] = self.clock()
                return s
            async with self._cond:
                try:
                    await asyncio.wait_for(self._cond.wait(), timeout=POLL)
                except asyncio.TimeoutError:
                    self.poll()

    async def leave(self, server: str):
        self.inflight[server] -= 1
        if self._cond is not None:
            async with self._cond:
                self._cond.notify_all()

    def state(self) -> dict:
        return {s: {"inflight": self.inflight[s], "trees": self.trees(s), "load": self.loads.get(s),
                    "slots": self.slots(s)} for s in self.servers}
