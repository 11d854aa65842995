"""Server-resident cursors: response id -> token sequence, KV slots and positions.

A cursor is what a finished reply leaves on the server: the full token sequence the
next request of the same thread continues from, the KV slots holding those tokens'
keys/values (shared zero-copy with whatever else holds them), the K2 position of each
row, and which rows are mounted (placeholders of another thread's segment).  A
continuation request sends only the new messages (``cursor`` + delta ids), and a
``mount`` splices a range of another cursor's rows into the context without copying
KV.  Entries live in an LRU under a byte budget (``OCTOPUS_CURSOR_BYTES``, default
2 GiB of host metadata); evicting an entry releases its slot references.  Under KV-pool
pressure the engine may instead *spill* a cursor (drop its KV, keep the entry and the
recipe that rebuilds it: ``Engine._spill`` / ``Engine._rebuild``).

Reference parity: `octopus/serving/cursor_store.py:27-81` (LRU cursor store under a
byte budget, position breakpoints, put_reply) and the placeholder convention of
`octopus/serving/kv_mount.py:87-138` (tokens(B) + placeholders(M_i) + delta).
"""
from __future__ import annotations

import os
import threading
from collections import OrderedDict
from dataclasses import dataclass, field

import numpy as np

PLACEHOLDER = -1  # token id of a mounted row inside a cursor's token sequence


@dataclass
class Cursor:
    cid: str
    tokens: np.ndarray      # int32 [L]; PLACEHOLDER for mounted rows
    slots: np.ndarray       # int64 [L] KV slot of each row
    positions: np.ndarray   # int64 [L] K2 position of each row
    prompt_len: int = 0     # rows that were prompt (the rest was generated)
    mounted: np.ndarray = field(default=None)  # bool [L] rows spliced in by a mount
    version: int = 0        # weight version the KV was computed under
    meta: dict = field(default_factory=dict)

    def __post_init__(self):
        if self.mounted is None:
            self.mounted = np.zeros(len(self.tokens), dtype=bool)

    @property
    def length(self) -> int:
        return int(len(self.tokens))

    @property
    def next_pos(self) -> int:
        return int(self.positions[-1]) + 1 if len(self.positions) else 0

    def nbytes(self) -> int:
        return int(self.tokens.nbytes + self.slots.nbytes + self.positions.nbytes + self.mounted.nbytes) + 128

    def held_slots(self) -> np.ndarray:
        """Slots this cursor references (rows without KV have slot -1)."""
        return self.slots[self.slots >= 0]

    def real_tokens(self) -> np.ndarray:
        return self.tokens[~self.mounted]


class CursorStore:
    """LRU of cursors; holds one pool reference per slot of every live cursor."""

    def __init__(self, pool=None, budget_bytes: int | None = None):
        self.pool = pool
        self.budget = budget_bytes if budget_bytes is not None else int(os.environ.get("OCTOPUS_CURSOR_BYTES",
                                                                                     2 << 30))
        self._d: OrderedDict[str, Cursor] = OrderedDict()
        self._bytes = 0
        self._lock = threading.Lock()
        self.evictions = 0

    def __contains__(self, cid):
        return cid in self._d

    def __len__(self):
        return len(self._d)

    def get(self, cid: str) -> Cursor | None:
        with self._lock:
            c = self._d.get(cid)
            if c is not None:
                self._d.move_to_end(cid)
            return c

    def peek(self, cid: str) -> Cursor | None:
        """The cursor without marking it recently used."""
        with self._lock:
            return self._d.get(cid)

    def oldest_first(self) -> list[str]:
        """Cursor ids from least to most recently used."""
        with self._lock:
            return list(self._d)

    def put(self, cur: Cursor, take_ref: bool = True) -> None:
        """Insert a cursor.  With take_ref the store adds its own reference to the slots."""
        with self._lock:
            if cur.cid in self._d:
                self._drop(cur.cid)
            if self.pool is not None and take_ref and len(cur.slots):
                self.pool.incref(cur.held_slots())
            self._d[cur.cid] = cur
            self._bytes += cur.nbytes()
            while self._bytes > self.budget and len(self._d) > 1:
                old = next(iter(self._d))
                self._drop(old)
                self.evictions += 1

    def pop(self, cid: str) -> None:
        with self._lock:
            if cid in self._d:
                self._drop(cid)

    def _drop(self, cid):
        c = self._d.pop(cid)
        self._bytes -= c.nbytes()
        if self.pool is not None and len(c.slots):
            self.pool.decref(c.held_slots())

    def clear(self):
        with self._lock:
            for cid in list(self._d):
                self._drop(cid)

    def nbytes(self) -> int:
        return self._bytes


def put_reply(store: CursorStore, cid: str, prompt: Cursor | None, new_tokens, new_slots, new_positions,
              generated, gen_slots, gen_positions, stop_ids=(), terminator=()) -> Cursor:
    """Record a finished reply as a cursor: prompt rows + new prompt delta + generated.

    Stop tokens at the end of the generation are stripped and the chat template's
    turn terminator ids are appended as plain tokens (they have no KV yet: their slots
    are -1 and the next continuation prefills them).
    """
    gen = list(generated)
    gsl = list(gen_slots)
    gps = list(gen_positions)
    while gen and gen[-1] in stop_ids:
        gen.pop()
        gsl.pop()
        gps.pop()
    toks = [] if prompt is None else [prompt.tokens]
    sl = [] if prompt is None else [prompt.slots]
    ps = [] if prompt is None else [prompt.positions]
    mt = [] if prompt is None else [prompt.mounted]
    toks += [np.asarray(new_tokens, np.int32), np.asarray(gen, np.int32)]
    sl += [np.asarray(new_slots, np.int64), np.asarray(gsl, np.int64)]
    ps += [np.asarray(new_positions, np.int64), np.asarray(gps, np.int64)]
    mt += [np.zeros(len(new_tokens) + len(gen), dtype=bool)]
    cur = Cursor(cid, np.concatenate(toks), np.concatenate(sl), np.concatenate(ps),
                 prompt_len=(0 if prompt is None else prompt.length) + len(new_tokens), mounted=np.concatenate(mt))
    store.put(cur)
    return cur
