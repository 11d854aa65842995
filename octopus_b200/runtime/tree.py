"""CursorRuntime: an episode's fork tree of threads, independent of the world they act in.

The main thread runs the agent loop (octopus_b200.runtime.core.run_thread).  A fork call
starts N branches, each a continuation of the forking thread's history plus a task
message, running concurrently as asyncio tasks in private workspaces (the provider's
copy); the forking thread's turn ends by joining them (their closing summaries become
a join note, committed results are applied by the provider).  Branches may fork again
below OCTOPUS_FORK_DEPTH; OCTOPUS_MAX_THREADS bounds threads running at once and
OCTOPUS_MAX_BRANCHES the branches per episode.  read_thread mounts another thread's
steps into the reader's context through the chat request's ``mount`` field (cursor
protocol), and every request is recorded (requests.jsonl rows: id, thread, prompt and
completion tokens, wall times) for credit assignment and critical-path costs.

Everything environment-specific is the WorkspaceProvider's.

Reference parity (behaviour): `octopus/runtime/tree.py:141-302` (WorkspaceProvider),
`tree.py:305-1440` (CursorRuntime: run, _complete, _thread_tool, _join, _start_fork,
_collect, _branch, _read, _write_tree).
"""
from __future__ import annotations

import asyncio
import itertools
import json
import os
import time
from pathlib import Path

from . import settings as S
from .core import (CLOSING, DONE_TOOL, READ_TOOL, RUNTIME_NAMES, RuntimePort, apply_runtime, branch_key,
                   branch_task_message, closing_name, closing_step, cursor_delta, handed, join_note, run_thread, runtime_tools,
                   thread_name, without_cursors)

FORK_DEPTH_REFUSAL = "Forking is not available at this depth; finish this task yourself."
FORK_WINDOW_REFUSAL = ("Forking is not available here: not enough context window is left at this depth; finish this "
                       "task yourself.")
FORK_THREADS_REFUSAL = "Forking is not available now: too many threads are running; finish this task yourself."
FORK_BRANCHES_REFUSAL = "Forking is not available: this episode has made all the branches it may."
ONE_FORK = "fork refused: one fork per reply, this reply's first fork call; put every task in that one fork's tasks."
MAIN_CLOSE = "{} has no effect in the main thread: a branch commits or aborts itself. End the main thread with done."
FORK_FLOOR = 8192
# a read that mounted: the source thread's full name, its steps (reply indices) and the rows mounted
MOUNT_RESULT = "read_thread: mounted {src} steps {a}-{b} ({n} tokens) into your attention from your next reply on"


class BranchCopyError(RuntimeError):
    pass


class WorkspaceProvider:
    """Environment hooks (override what the environment has; defaults: no workspace)."""

    report = "findings, files, changes"

    def system_prompt(self, task: str) -> str:
        return "You are an agent. Use the tools. Call done with the answer when finished."

    def tools(self) -> list[dict]:
        return [DONE_TOOL]

    def budget(self) -> int | None:
        """Shared completion-token budget of the whole episode (None: none)."""
        return None

    def closing(self, depth: int) -> set:
        return {"done"} if depth == 0 else {"commit", "abort"}

    def fork_min(self) -> int:
        return 2

    async def dispatch(self, name: str, args: dict, thread: str) -> tuple[str, bool]:
        if name == "done":
            return f"done: {args.get('answer', '')}", True
        return f"unknown tool {name}", False

    async def copy(self, parent: str, child: str) -> None:
        return None

    async def snapshot(self, thread: str):
        return None

    async def restore(self, thread: str, snap) -> None:
        return None

    async def capture(self, thread: str) -> dict:
        return {}

    async def apply(self, thread: str, results: list[dict]) -> str:
        return ""

    async def check_close(self, start: dict, args: dict, closes: bool, run) -> tuple[str | None, dict]:
        return None, {}

    async def close(self) -> None:
        return None


class CursorRuntime:
    """Runs one episode.  `complete(body) -> payload` is the chat transport (async or sync):
    body = {"messages", "tools", "session_id", "cursor"?, "mount"?}; payload in the OpenAI
    shape with "id", "usage", and optionally "cursor"."""

    def __init__(self, ws: WorkspaceProvider, complete, *, session_id: str = "ep", log_dir: str | None = None,
                 max_main_calls: int | None = None, branch_turns: int | None = None):
        self.ws = ws
        self._complete_fn = complete
        self.session_id = session_id
        self.log_dir = Path(log_dir) if log_dir else None
        self.max_main_calls = max_main_calls if max_main_calls is not None else S.call_limit()
        self.branch_turns = branch_turns if branch_turns is not None else S.branch_turns()
        self.cursor = S.cursor_mode()
        self.requests: list[dict] = []
        self.threads: dict[str, dict] = {}  # thread -> {"steps", "replies": [(id, prompt_tokens, completion)]}
        self.forks: dict[str, list] = {"main": []}
        self.branches_made = 0
        self.running = 1
        self.used = 0  # completion tokens against the shared budget
        self.budget_out = False
        self.pending_mounts: dict[str, list] = {}
        self._read_caps: dict[str, dict] = {}  # OCTOPUS_READ_CONTROL: branch -> state before its mount request
        self._ids = itertools.count()

    # ------------------------------------------------------------------ transport
    async def _complete(self, thread: str, messages: list, session_id: str) -> dict:
        body = {"messages": messages, "tools": self.tool_list(thread), "session_id": session_id,
                "max_tokens": S.max_reply()}
        if self.cursor:
            cur, delta = cursor_delta(messages)
            if cur is not None:
                body["cursor"], body["messages"] = cur, delta
                if os.environ.get("OCTOPUS_CURSOR_AUDIT"):
                    body["audit_messages"] = without_cursors(messages)
        if self.pending_mounts.get(thread):
            body["mount"] = list(self.pending_mounts[thread])
            if S.read_control() and self._is_branch(thread) and thread not in self._read_caps:
                await self._capture_read(thread, messages)
        t0 = time.time()
        payload = self._complete_fn(body)
        if hasattr(payload, "__await__"):
            payload = await payload
        usage = payload.get("usage") or {}
        rid = payload.get("id") or f"{session_id}-{next(self._ids)}"
        payload.setdefault("id", rid)
        row = {"id": rid, "thread": thread, "t": t0, "elapsed_s": round(time.time() - t0, 4),
               "prompt_tokens": int(usage.get("prompt_tokens") or 0),
               "completion_tokens": int(usage.get("completion_tokens") or 0),
               "cached_tokens": int((usage.get("prompt_tokens_details") or {}).get("cached_tokens") or 0),
               "mounted": len(body.get("mount") or [])}
        self.requests.append(row)
        self.threads.setdefault(thread, {"replies": []})["replies"].append(
            (rid, row["prompt_tokens"], row["completion_tokens"], payload.get("cursor")))
        budget = self.ws.budget()
        if budget:
            self.used += row["completion_tokens"]
            if self.used >= budget:
                self.budget_out = True
                payload["budget_out"] = True
        return payload

    def tool_list(self, thread: str) -> list[dict]:
        tools = self.ws.tools() + runtime_tools()
        if S.read_tool():
            tools = tools + [READ_TOOL]
        return tools

    # ------------------------------------------------------------------ threads
    def depth(self, thread: str) -> int:
        return 0 if thread == "main" else thread.count("fork")

    async def _thread_tool(self, thread: str, port: RuntimePort, forks_this_turn: list, name: str, args: dict):
        depth = self.depth(thread)
        if name == "fork":
            if thread == "control" or thread.startswith("readctl/"):  # controls run without forks
                return FORK_DEPTH_REFUSAL, False
            if forks_this_turn:
                return ONE_FORK, False
            if thread == "main" and getattr(self, "_control_snap", None) is None and S.plan_control():
                self._control_snap = await self.ws.snapshot("main")  # main's workspace at its first fork
            if depth >= S.fork_depth():
                return FORK_DEPTH_REFUSAL, False
            cap = S.max_branches()
            if cap is not None and self.branches_made >= cap:
                return FORK_BRANCHES_REFUSAL, False
            if self.running >= S.max_threads():
                return FORK_THREADS_REFUSAL, False
            replies = self.threads.get(thread, {}).get("replies") or []
            ctx = (replies[-1][1] + replies[-1][2]) if replies else 0
            if S.window_room(ctx) < FORK_FLOOR + S.answer_reserve():
                return FORK_WINDOW_REFUSAL, False
            obs, stop = apply_runtime("fork", args, port, fewest=self.ws.fork_min())
            if port.last_fork and obs.startswith("fork started"):
                forks_this_turn.append(port.last_fork)
                self.branches_made += len(port.last_fork["branches"])
            return obs, stop
        if name in ("commit", "abort"):
            if depth == 0:
                return MAIN_CLOSE.format(name), False
            return apply_runtime(name, args, port)
        if name == "read_thread":
            if thread.startswith("readctl/"):  # a read control runs without the mount it replaces
                return "read_thread: not available in this thread", False
            return self._read(thread, args), False
        return await self.ws.dispatch(name, args, thread)

    def _read(self, reader: str, args: dict) -> str:
        """Mount steps [from_step, to_step] of another thread into the reader's next requests."""
        target = args.get("thread")
        names = {t: t for t in self.threads} | {t.rsplit("/", 1)[-1]: t for t in self.threads if t != "main"}
        src = names.get(target)
        if src == reader:
            return "read_thread: a thread reads other threads, never itself"
        if src is None:
            return f"read_thread: no other thread named {target!r}"
        replies = self.threads[src]["replies"]
        if not replies or replies[-1][3] is None:
            return f"read_thread: {target} has no readable step yet"
        n = len(replies)
        a = args.get("from_step")
        b = args.get("to_step")
        a = 0 if a is None else max(0, int(a))
        b = n - 1 if b is None else min(n - 1, int(b))
        if a > b:
            return "read_thread: from_step must not be after to_step"
        cursor = replies[-1][3]
        start_tok = replies[a][1]
        end_tok = replies[b][1] + replies[b][2] - 1  # rows with KV: all but the last sampled token
        if end_tok <= start_tok:
            return "read_thread: nothing readable in that range"
        self.pending_mounts.setdefault(reader, []).append((cursor, start_tok, end_tok))
        return MOUNT_RESULT.format(src=src, a=a, b=b, n=end_tok - start_tok)

    async def _run_thread(self, thread: str, start: dict, depth: int, max_steps_left: int | None = None) -> dict:
        port = RuntimePort(owner=None if thread == "main" else start["branch_id"])
        forks_this_turn: list = []
        my_forks = self.forks.setdefault(thread, [])

        async def dispatch(name, args, bid):
            return await self._thread_tool(thread, port, forks_this_turn, name, args)

        async def complete(messages, sid):
            forks_this_turn.clear()
            return await self._complete(thread, messages, sid)

        async def join(messages):
            if not forks_this_turn:
                return None
            fork = forks_this_turn[0]
            record = {"response_id": self.threads[thread]["replies"][-1][0], "branches": [],
                      "prefix_len": len(messages)}  # the parent's history at the fork (its join note follows)
            my_forks.append(record)
            k = len(my_forks) - 1
            tasks = []
            for br in fork["branches"]:
                child = thread_name(thread, k, br["branch_id"])
                try:
                    await self.ws.copy(thread, child)
                except BranchCopyError as e:
                    record["branches"].append({"branch_id": br["branch_id"], "task": br["task"],
                                               "ended_with": "copy failed", "error": str(e)})
                    continue
                hist = without_cursors(messages) if not self.cursor else list(messages)
                msg = branch_task_message(br["branch_id"], br["task"], len(fork["branches"]), self.ws.report)
                bstart = {"branch_id": br["branch_id"], "session_id": f"{self.session_id}/{child}",
                          "task": br["task"], "messages": hist + [{"role": "user", "content": msg}],
                          "step": start.get("step")}
                self.running += 1
                tasks.append((br, child, len(bstart["messages"]),
                              asyncio.ensure_future(self._run_thread(child, bstart, depth + 1))))
            results = []
            for br, child, prefix_len, t in tasks:
                try:
                    res = await t
                finally:
                    self.running -= 1
                cl = closing_step(res["steps"])
                out = {"branch_id": br["branch_id"], "task": br["task"], "thread": child,
                       "ended_with": closing_name(res["steps"]) if cl else "stopped",
                       "summary": handed(cl), "end_time": time.time(), "forks": self.forks.get(child, []),
                       "result": await self.ws.capture(child),
                       # the branch's history (inherited prefix + its own turns) for offline analysis
                       "messages": without_cursors(res["messages"]), "prefix_len": prefix_len,
                       "rewinds": len(res.get("rewinds") or []), "tools": self.tool_list(child)}
                record["branches"].append(out)
                results.append(out)
            record["join_response_id"] = record["response_id"]
            applied = await self.ws.apply(thread, results)
            note = join_note(results)
            return note + ("\n" + applied if applied else "")

        closing = self.ws.closing(depth)
        max_steps = None if depth == 0 else self.branch_turns
        if max_steps_left is not None:
            max_steps = max_steps_left if max_steps is None else min(max_steps, max_steps_left)
        max_calls = self.max_main_calls if depth == 0 else None
        budget = S.thread_budget()

        def before_turn(turns):
            return "budget used up" if self.budget_out else None

        res = await run_thread(start, complete, dispatch, max_steps=max_steps, closing=closing, budget=budget,
                               join=join, max_calls=max_calls, before_turn=before_turn,
                               snapshot=lambda: self.ws.snapshot(thread),
                               restore=lambda snap: self.ws.restore(thread, snap), ws=self.ws)
        self.threads.setdefault(thread, {"replies": []}).update(steps=res["steps"], messages=res["messages"])
        return res

    # ------------------------------------------------------------------ episode
    async def run(self, task: str) -> dict:
        start = {"branch_id": "main", "session_id": self.session_id, "task": task,
                 "messages": [{"role": "system", "content": self.ws.system_prompt(task)},
                              {"role": "user", "content": task}]}
        self._control_snap = None
        res = await self._run_thread("main", start, 0)
        tree = {"task": task, "tools": self.tool_list("main"), "forks": self.forks.get("main", []),
                "main_end": self._main_end(res["steps"]),
                "answer": handed(closing_step(res["steps"])), "requests": len(self.requests),
                "budget": self.ws.budget(), "used": self.used, "reminded": res["reminded"]}
        if S.plan_control() and tree["forks"]:
            tree["control"] = await self._control(task, res)
        if S.read_control() and self._read_caps:
            tree["read_controls"] = [await self._read_control(task, th, cap) for th, cap in self._read_caps.items()]
        if self.log_dir:
            self._write(tree, res)
        await self.ws.close()
        return {"tree": tree, "main": res, "requests": self.requests}

    async def _control(self, task: str, main_res: dict) -> dict:
        """The main-first control: main's history up to (not including) its first forking
        reply, continued without forks (fork is refused) in a copy of main's workspace at that
        point, with the calls main had left; closed by done like main.  Its requests are
        logged under thread "control" (never trained); the record gives its answer."""
        msgs = main_res["messages"]
        pl = int(self.forks["main"][0].get("prefix_len", len(msgs)))
        idx = max((i for i in range(min(pl, len(msgs))) if msgs[i].get("role") == "assistant"), default=None)
        if idx is None:
            return {"kind": "main-first", "error": "no forking reply"}
        ctrl = [dict(m) for m in msgs[:idx]]
        calls_before = sum(1 for m in ctrl if m.get("role") == "assistant")
        try:
            await self.ws.copy("main", "control")
            if self._control_snap is not None:
                await self.ws.restore("control", self._control_snap)
        except BranchCopyError as e:
            return {"kind": "main-first", "error": f"copy failed: {e}"}
        saved = self.max_main_calls
        if saved is not None:
            self.max_main_calls = max(1, saved - calls_before)
        start = {"branch_id": "control", "session_id": f"{self.session_id}/control", "task": task, "messages": ctrl}
        n0 = len(self.requests)
        try:
            res = await self._run_thread("control", start, 0)
        finally:
            self.max_main_calls = saved
        return {"kind": "main-first", "calls_before": calls_before, "answer": handed(closing_step(res["steps"])),
                "main_end": self._main_end(res["steps"]), "requests": len(self.requests) - n0}

    # ------------------------------------------------------------------ read controls
    @staticmethod
    def _is_branch(thread: str) -> bool:
        return thread not in ("main", "control") and not thread.startswith("readctl/")

    async def _capture_read(self, thread: str, messages: list) -> None:
        """OCTOPUS_READ_CONTROL: the state just before a branch's first request that carries a
        mount: its history, its workspace, the reply whose read_thread call mounted and the
        turns it had used.  _read_control continues from here without the mount."""
        reply = next((m for m in reversed(messages) if m.get("role") == "assistant"), {})
        names = [(c.get("function") or {}).get("name") for c in reply.get("tool_calls") or []]
        results = [str(m.get("content") or "") for m in messages if m.get("role") == "tool"][-len(names):] \
            if names else []
        reads = [k for k, n in enumerate(names) if n == "read_thread"]
        mounted = [j for j, k in enumerate(reads) if k < len(results) and results[k].startswith("read_thread: mounted")]
        replies = self.threads.get(thread, {}).get("replies") or []
        self._read_caps[thread] = {
            "messages": [dict(m) for m in messages], "snap": await self.ws.snapshot(thread),
            "read_rid": replies[-1][0] if replies else None, "read_calls": names,
            "read_call": mounted[0] if mounted else 0, "turns": len(replies), "history": len(messages)}

    async def _read_control(self, task: str, thread: str, cap: dict) -> dict:
        """One read control: the reader's state before its mount request continued without the
        mount (forks and reads refused), in a copy of the reader's workspace restored to that
        point, with the turns the reader had left.  Its requests are logged under thread
        readctl/<reader> (never trained); the record names the reader (`of`, the branch key),
        the read reply and call, how the control ended and its result for grading."""
        name = f"readctl/{thread}"
        rec = {"of": branch_key(thread), "thread": thread, "read_rid": cap["read_rid"], "read_calls": cap["read_calls"],
               "read_call": cap["read_call"]}
        later = (self.threads.get(thread, {}).get("messages") or [])[cap["history"]:]
        rec["forked_after"] = any((c.get("function") or {}).get("name") == "fork"
                                  for m in later if m.get("role") == "assistant" for c in m.get("tool_calls") or [])
        try:
            await self.ws.copy(thread, name)
            if cap["snap"] is not None:
                await self.ws.restore(name, cap["snap"])
        except BranchCopyError as e:
            return {**rec, "error": f"copy failed: {e}"}
        bid = thread.rsplit("/", 1)[-1]
        start = {"branch_id": bid, "session_id": f"{self.session_id}/{name}", "task": task,
                 "messages": [dict(m) for m in cap["messages"]]}
        left = None if self.branch_turns is None else max(1, self.branch_turns - cap["turns"])
        n0 = len(self.requests)
        res = await self._run_thread(name, start, self.depth(thread), max_steps_left=left)
        closing = closing_step(res["steps"])
        rec.update(end=closing_name(res["steps"]) if closing else "stopped", summary=handed(closing),
                   control_forked=any(s.get("name") == "fork" for s in res["steps"]),
                   requests=len(self.requests) - n0, result=await self.ws.capture(name))
        return rec

    def _main_end(self, steps: list) -> str:
        if any(s.get("name") == "done" and not s.get("rejected") for s in steps):
            return "done"
        if self.budget_out:
            return "budget"
        last = steps[-1] if steps else {"name": None, "text": ""}
        if last.get("name"):
            return "context" if last["name"] == "context" else "step cap"
        t = str(last.get("text") or "")
        return "step cap" if t.startswith("stopped: ") else "request failed" if t.startswith("request failed") \
            else "no tool call"

    def _write(self, tree: dict, res: dict) -> None:
        d = self.log_dir
        d.mkdir(parents=True, exist_ok=True)
        (d / "tree.json").write_text(json.dumps(without_cursors({**tree, "main": res["messages"]}), indent=1,
                                                default=str))
        (d / "trajectory.json").write_text(json.dumps(without_cursors(res["messages"]), indent=1, default=str))
        with open(d / "requests.jsonl", "w") as f:
            for r in self.requests:
                f.write(json.dumps(r) + "\n")


def run_episode(ws: WorkspaceProvider, complete, task: str, **kw) -> dict:
    """Synchronous helper: run one episode to completion."""
    return asyncio.run(CursorRuntime(ws, complete, **kw).run(task))
