"""Engine hop: the client side of the cursor protocol over a pool of engine servers.

A reply lives as a cursor on the server that produced it.  `EngineHop.generate` sends a
continuation to its parent cursor's server with only the new token ids (the "hop"
saves resending the history), and mounts rows of other replies with offsets adjusted
for the placeholder rows that earlier mounts inserted into those replies' cursors
(callers address a reply's visible tokens; the server addresses cursor rows).  When the
server no longer knows the parent (404: evicted, restarted), the full visible history is
resent without a cursor, unless the history holds mounted rows (they cannot be
re-rendered from text) — then the error propagates.  Every response's prompt size is
checked against the rows the client expects, and the new reply's server, visible
history and placeholder runs are recorded.

Reference parity (behaviour): `patches/areal-cursor.patch:371-540` (the AReaL engine
hop: parent routing, cursor + delta ids, placeholder-adjusted mounts, resend on 404
unless mounted, prompt_tokens verification).
"""
from __future__ import annotations

import json
import urllib.error
import urllib.request


class HopError(RuntimeError):
    pass


def http_transport(server: str, path: str, body: dict, timeout: float = 600.0):
    req = urllib.request.Request(f"http://{server}{path}", data=json.dumps(body).encode(),
                                 headers={"Content-Type": "application/json"})
    try:
        with urllib.request.urlopen(req, timeout=timeout) as r:
            return getattr(r, "status", 200), json.loads(r.read().decode())
    except urllib.error.HTTPError as e:
        return e.code, {"error": e.read().decode("utf-8", "replace")[:300]}


class EngineHop:
    def __init__(self, servers: list[str], transport=None, pick=None):
        if not servers:
            raise ValueError("no servers")
        self.servers = list(servers)
        self.transport = transport or http_transport
        self.pick = pick or (lambda session: self.servers[hash(session) % len(self.servers)])
        self.where: dict[str, str] = {}        # reply cursor -> server
        self.visible: dict[str, list] = {}     # reply cursor -> visible token history (prompt + output)
        self.runs: dict[str, list] = {}        # reply cursor -> [(row, n)] placeholder runs in its rows
        self.stats = {"hops": 0, "resent": 0, "bytes_sent": 0, "bytes_saved": 0}

    # ------------------------------------------------------------------ offsets
    def rows(self, cursor: str, v0: int, v1: int) -> tuple[int, int]:
        """Visible token range [v0, v1) of a reply -> its cursor rows (must not split a run)."""
        def row(v):
            r = v
            for at, n in self.runs.get(cursor, []):
                if at <= r:
                    r += n
            return r
        return row(v0), row(v1 - 1) + 1 if v1 > v0 else row(v0)

    def _rows_total(self, cursor: str) -> int:
        return len(self.visible[cursor]) + sum(n for _, n in self.runs.get(cursor, []))

    # ------------------------------------------------------------------ request
    def generate(self, ids: list[int], parent: str | None = None, mount=(), sampling: dict | None = None,
                 session: str = "") -> dict:
        mount = list(mount)
        server = self.where.get(parent) if parent else None
        for src, _, _ in mount:
            s = self.where.get(src)
            if s is None:
                raise HopError(f"mount source {src} unknown to this client")
            if server is not None and s != server:
                raise HopError(f"mount source {src} lives on {s}, the parent on {server}")
            server = server or s
        server = server or self.pick(session)
        m_rows = [(src, *self.rows(src, a, b)) for src, a, b in mount]
        body = {"input_ids": list(ids), "sampling_params": dict(sampling or {})}
        if parent:
            body["cursor"] = parent
        if m_rows:
            body["mount"] = [{"cursor": c, "start": a, "end": b} for c, a, b in m_rows]
        base_rows = self._rows_total(parent) if parent else 0
        expect = base_rows + len(ids)  # the server counts cursor rows + new ids (this request's mounts are free)
        status, out = self.transport(server, "/generate", body)
        self.stats["hops"] += 1
        self.stats["bytes_sent"] += len(json.dumps(body))
        if parent:
            self.stats["bytes_saved"] += 8 * len(self.visible.get(parent, []))
        if status == 404 and parent:
            if self.runs.get(parent) or m_rows:
                raise HopError(f"cursor {parent} is gone on {server} and its history holds mounted rows")
            full = self.visible[parent] + list(ids)
            body = {"input_ids": full, "sampling_params": dict(sampling or {})}
            status, out = self.transport(server, "/generate", body)
            self.stats["resent"] += 1
            expect, parent, ids = len(full), None, full
            base_rows = 0
        if status != 200:
            raise HopError(f"generate on {server}: HTTP {status} {out.get('error', '')}")
        meta = out["meta_info"]
        got = int(meta["prompt_tokens"]) + int(meta["cached_tokens"])
        if got != expect:
            raise HopError(f"server counted {got} prompt rows, the client expects {expect}")
        cid = meta.get("cursor")
        if cid:
            hist = (self.visible[parent] if parent else []) + list(ids) + list(out["output_ids"])
            runs = list(self.runs.get(parent, [])) if parent else []
            at = base_rows
            for _, a, b in m_rows:  # mounted rows sit after the parent's rows, before the new ids
                runs.append((at, b - a))
                at += b - a
            self.where[cid], self.visible[cid], self.runs[cid] = server, hist, runs
        out["cursor"] = cid
        out["placeholders"] = sum(n for _, n in self.runs.get(cid, [])) if cid else 0
        return out

    def release(self, cursor: str):
        s = self.where.pop(cursor, None)
        self.visible.pop(cursor, None)
        self.runs.pop(cursor, None)
        if s is not None:
            self.transport(s, "/release_cursor", {"cursor": cursor})
