"""In-process chat service over the engine: request scheduling (continuous batching, or
static windows for engines without it), chat rendering with the
cursor protocol (only the messages after the cursor's reply are rendered), tool-call
parsing, and the template terminator kept on the reply's cursor.  The HTTP server wraps
it; the RL agent environment calls it directly as the runtime's completion function
(no HTTP hop for colocated rollouts).

OCTOPUS_CURSOR_AUDIT=<path>: for every cursor request that carries the full history in
``audit_messages``, append a JSONL row comparing the assembled prompt with the oracle.

Reference parity (behaviour): `octopus/serving/cursor_audit.py:30-59` (audit rows); the AReaL proxy the reference runs in-process
(`octopus/rl/proxy.py:32-78`) and the chat path of `patches/apply_sglang_cursor.py`.
"""
from __future__ import annotations

import asyncio
import json
import os
import threading
import time
import uuid

from .chat import ChatTokenizer, parse_tool_calls
from .engine import Engine, GenInput


def mounts_of(body: dict) -> list:
    out = []
    for m in body.get("mount") or []:
        if isinstance(m, dict):
            out.append((m["cursor"], int(m["start"]), int(m["end"])))
        else:
            out.append((m[0], int(m[1]), int(m[2])))
    return out


class BatchingQueue:
    """Static batching for engines without continuous batching (hybrid and tensor-parallel
    engines): collects concurrent requests for `window` seconds and runs them as one engine
    batch per sampling setting.  A failing batch is retried request by request, so one bad
    request (unknown cursor, bad mount) fails alone."""

    def __init__(self, engine: Engine, window: float = 0.005, max_batch: int | None = None):
        self.engine = engine
        self.window = window
        self.max_batch = max_batch or engine.max_batch
        self.pending: list = []
        self.inflight = 0
        self.run_lock = asyncio.Lock()

    @property
    def n_waiting(self) -> int:
        return len(self.pending)

    @property
    def n_running(self) -> int:
        return self.inflight

    async def _run_group(self, loop, items):
        try:
            outs = await loop.run_in_executor(None, self.engine.generate, [i for i, _ in items])
        except Exception:  # noqa: BLE001  (isolate the failing request)
            if len(items) == 1:
                raise
            for item in items:
                try:
                    await self._run_group(loop, [item])
                except Exception as e:  # noqa: BLE001
                    if not item[1].done():
                        item[1].set_exception(e)
            return
        for (_, f), o in zip(items, outs):
            f.set_result(o)

    async def submit(self, inp: GenInput):
        loop = asyncio.get_running_loop()
        fut = loop.create_future()
        self.pending.append((inp, fut))
        self.inflight += 1
        await asyncio.sleep(self.window)
        async with self.run_lock:
            batch = [(i, f) for i, f in self.pending if not f.done()][: self.max_batch]
            if batch and not fut.done():
                for item in batch:
                    self.pending.remove(item)
                # one sampling setting per engine batch: group by (temperature, top_p, top_k)
                groups: dict = {}
                for i, f in batch:
                    groups.setdefault((float(i.temperature), float(i.top_p), int(i.top_k)), []).append((i, f))
                for items in groups.values():
                    try:
                        await self._run_group(loop, items)
                    except Exception as e:  # noqa: BLE001
                        for _, f in items:
                            if not f.done():
                                f.set_exception(e)
        try:
            return await fut
        finally:
            self.inflight -= 1


class ContinuousQueue:
    """The engine's continuous-batching scheduler (serving.scheduler) behind an async API."""

    def __init__(self, engine: Engine):
        from .scheduler import Scheduler

        self.engine = engine
        self.sched = Scheduler(engine)

    @property
    def n_waiting(self) -> int:
        return self.sched.pending

    @property
    def n_running(self) -> int:
        return self.sched.running

    async def submit(self, inp: GenInput):
        return await asyncio.wrap_future(self.sched.submit(inp))

    def close(self):
        self.sched.close()


def make_queue(engine: Engine, window: float = 0.005):
    """Continuous batching where the engine supports it (OCTOPUS_STATIC_BATCHING=1: static
    windows everywhere), else static windows."""
    if getattr(engine, "supports_continuous", False) and os.environ.get("OCTOPUS_STATIC_BATCHING", "0") != "1":
        return ContinuousQueue(engine)
    return BatchingQueue(engine, window)


def _top_k(v) -> int:
    """OpenAI / SGLang top_k: absent, None, 0 or -1 mean no top-k."""
    return 0 if v is None or int(v) < 0 else int(v)


class ChatService:
    """OpenAI-style chat completions (+ cursor / mount) on an engine, batched."""

    def __init__(self, engine: Engine, tokenizer: ChatTokenizer, model_name: str = "octopus-b200",
                 window: float = 0.005, tool_format: str | None = None):
        from .tool_parsers import detect_format

        self.engine, self.tok, self.model_name = engine, tokenizer, model_name
        # the tool-call markup the model emits: given, else the chat template's family
        self.tool_format = tool_format or detect_format(tokenizer.template_src)
        self.q = make_queue(engine, window)
        self._audit_lock = threading.Lock()

    async def chat(self, body: dict) -> dict:
        tok = self.tok
        msgs = body.get("messages") or []
        tools = body.get("tools")
        kwargs = body.get("chat_template_kwargs") or {}
        cursor = body.get("cursor")
        ids = tok.render_delta(msgs, tools, **kwargs) if cursor is not None else tok.apply(msgs, tools, True, **kwargs)
        audit = os.environ.get("OCTOPUS_CURSOR_AUDIT")
        if audit and cursor is not None and body.get("audit_messages") and not body.get("mount"):
            self._audit(audit, body, cursor, ids, tools, kwargs)
        inp = GenInput(ids, cursor=cursor, mount=mounts_of(body), max_new_tokens=int(body.get("max_tokens", 1024)),
                       temperature=float(body.get("temperature", 1.0)), stop_ids=tok.stop_ids,
                       top_p=float(body.get("top_p", 1.0)), top_k=_top_k(body.get("top_k")))
        o = await self.q.submit(inp)
        out_ids = [t for t in o.output_ids if t not in tok.stop_ids]
        content, calls = parse_tool_calls(tok.decode(out_ids), self.tool_format, tools)
        # the cursor keeps reply tokens + template terminator so the next delta renders right after it
        eng = self.engine
        if o.cursor is not None and eng.cursors.get(o.cursor) is not None:
            eng.extend_cursor(o.cursor, tok.terminator(), drop_trailing=tok.stop_ids)
        rid = o.cursor or f"chatcmpl-{uuid.uuid4().hex[:12]}"
        return {
            "id": rid, "object": "chat.completion", "created": int(time.time()), "model": self.model_name,
            "cursor": o.cursor,
            "choices": [{"index": 0, "finish_reason": "tool_calls" if calls else o.finish_reason,
                         "message": {"role": "assistant", "content": content, "tool_calls": calls or None}}],
            "usage": {"prompt_tokens": o.prompt_tokens + o.cached_tokens, "completion_tokens": len(o.output_ids),
                      "prompt_tokens_details": {"cached_tokens": o.cached_tokens}},
        }

    def _audit(self, path: str, body: dict, cursor: str, delta_ids: list, tools, kwargs):
        """Cursor audit: the prompt the engine assembles (cursor tokens + rendered delta)
        against rendering the whole conversation (the oracle), with the bytes the hop saved."""
        cur = self.engine.cursors.get(cursor)
        if cur is None:
            return
        full = self.tok.apply(body["audit_messages"], tools, True, **kwargs)
        assembled = [int(t) for t in cur.tokens] + list(delta_ids)
        row = {"t": time.time(), "cursor": cursor, "equal": assembled == full, "assembled_tokens": len(assembled),
               "oracle_tokens": len(full),
               "first_diff": next((i for i, (a, b) in enumerate(zip(assembled, full)) if a != b),
                                  None if len(assembled) == len(full) else min(len(assembled), len(full))),
               "hop_bytes": len(json.dumps(body.get("messages") or [])),
               "full_bytes": len(json.dumps(body["audit_messages"]))}
        with self._audit_lock:
            with open(path, "a") as f:
                f.write(json.dumps(row) + "\n")

    __call__ = chat
