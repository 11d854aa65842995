"""Runtime core: tool-call formats, the chat transport and cursor protocol, thread
names, the runtime tools (fork / commit / abort / done / rewind / read_thread) and one
thread's loop until it closes.

Everything environment-specific (workspace, working tools, grading) belongs to a
WorkspaceProvider (octopus_b200.runtime.tree).  Switches: octopus_b200.runtime.settings.

Reference parity (behaviour): `octopus/runtime/core.py:33-56` (TOOL_FORMATS per tool-call
parser), `core.py:84-112` (cursor_delta / with_cursor / without_cursors), `core.py:129-198`
(post_chat with retry/backoff on 403/429/5xx), `core.py:252-388` (runtime tools,
RuntimePort, apply_runtime with lenient task parsing), `core.py:508-777` (thread loop:
turn/call caps, growth budget and window room, answer reserve, remind-once,
FORK_ALONE, rewind tool), `core.py:817-1058` (branch task message, join note, fork
record).  The loop here is a re-implementation of those rules, not of their code.
"""
from __future__ import annotations

import bisect
import collections
import itertools
import json
import os
import re
import time
import urllib.error
import urllib.request
from dataclasses import dataclass, field

from . import settings as S

# How models write tool calls, per tool-call parser (group `name` = tool name, or `json`
# = the opening brace of a JSON call object whose "name" is the tool).
TOOL_FORMATS = {
    "qwen3_coder": {"call": r"<function=(?P<name>[^>\n]+)>.*?</function>"},
    "qwen25": {"call": r"<tool_call>\s*(?P<json>\{)"},
    "llama3": {"call": r"(?:^|<\|python_tag\|>|<\|end_header_id\|>|;)\s*(?P<json>\{)"},
    "mistral": {"call": r"\[TOOL_CALLS\](?P<name>[^\[\s]+)(?:\[CALL_ID\][^\[]*)?\[ARGS\]\{.*?\}"
                        r"(?=\s*(?:\[TOOL_CALLS\]|</s>|$))|(?:\[TOOL_CALLS\]\s*\[|(?<=\}),)\s*(?P<json>\{)"},
    "deepseekv3": {"call": r"<｜tool▁call▁begin｜>function<｜tool▁sep｜>(?P<name>[^\n]+)\n.*?<｜tool▁call▁end｜>"},
    "deepseekv31": {"call": r"<｜tool▁call▁begin｜>(?P<name>[^<]+)<｜tool▁sep｜>.*?<｜tool▁call▁end｜>"},
    "glm45": {"call": r"<tool_call>(?P<name>[^\n<]+).*?</tool_call>"},
    "kimi_k2": {"call": r"<\|tool_call_begin\|>\s*(?:functions\.)?(?P<name>[\w.\-]+):\d+\s*"
                        r"<\|tool_call_argument_begin\|>.*?<\|tool_call_end\|>"},
    "gpt-oss": {"call": r"to=functions\.(?P<name>[^\s<]+).*?<\|call\|>"},
}
for _alias, _target in (("qwen", "qwen25"), ("hermes", "qwen25"), ("step3p5", "qwen3_coder"), ("glm", "glm45"),
                        ("glm47", "glm45")):
    TOOL_FORMATS[_alias] = TOOL_FORMATS[_target]


def tool_format(name: str = "") -> dict:
    name = name or S.tool_format_name()
    if name not in TOOL_FORMATS:
        raise ValueError(f"tool-call format {name!r} is none of {sorted(TOOL_FORMATS)}")
    return TOOL_FORMATS[name]


def token_index(pieces: list[str]):
    """Token texts -> (joined text, char offset -> index of the token covering it)."""
    ends = list(itertools.accumulate(len(p) for p in pieces))
    return "".join(pieces), lambda off: bisect.bisect_right(ends, off)


_JSON = json.JSONDecoder()


def tool_calls_in_text(text: str, fmt: str = "") -> list[tuple[str, int, int]]:
    """(name, start, end) of each tool call written in `text` (the run's tool-call format)."""
    out, end = [], 0
    for m in re.finditer(tool_format(fmt)["call"], text, re.S):
        if m.groupdict().get("name"):
            out.append((m.group("name"), m.start(), m.end()))
        elif m.start() >= end:
            try:
                call, end = _JSON.raw_decode(text, m.start("json"))
            except json.JSONDecodeError:
                continue
            if isinstance(call, dict) and isinstance(call.get("name"), str):
                out.append((call["name"], m.start("json"), end))
    return out


# ---------------------------------------------------------------------------- cursor protocol
def reply_tools(choice: dict) -> tuple[list, str]:
    return choice.get("tool_calls") or [], choice.get("content") or ""


def reply_message(choice: dict, content, tool_calls: list | None = None) -> dict:
    msg = {"role": "assistant", "content": content}
    if tool_calls is not None:
        msg["tool_calls"] = tool_calls
    if choice.get("reasoning_content"):
        msg["reasoning_content"] = choice["reasoning_content"]
    return msg


def cursor_delta(messages: list[dict]) -> tuple[str | None, list[dict]]:
    """What a cursor-mode request sends: (the cursor of the newest message that carries
    one, the messages after it), or (None, every message) when none carries a cursor."""
    marked = [i for i, m in enumerate(messages) if "cursor" in m]
    if not marked:
        return None, messages
    last = marked[-1]
    return messages[last]["cursor"], messages[last + 1:]


def with_cursor(reply: dict, payload: dict) -> dict:
    """Mark the reply with the response's cursor only if it is kept exactly as the server sent it."""
    if "cursor" not in payload:
        return reply
    ch = payload["choices"][0]["message"]
    if (reply.get("content") or "") == (ch.get("content") or "") and \
            reply.get("tool_calls") == (ch.get("tool_calls") or None):
        reply["cursor"] = payload["cursor"]
    return reply


def without_cursors(value):
    if isinstance(value, dict):
        return {k: without_cursors(v) for k, v in value.items() if k != "cursor"}
    if isinstance(value, list):
        return [without_cursors(v) for v in value]
    return value


def decode_tool_call(call: dict, default_id: str = "") -> tuple[str, dict, str]:
    fn = call.get("function") or {}
    name = fn.get("name") or "shell"
    raw = fn.get("arguments") or "{}"
    try:
        args = json.loads(raw) if isinstance(raw, str) else raw
    except (json.JSONDecodeError, TypeError):
        args = {"command": str(raw)}
    if not isinstance(args, dict):
        args = {"command": str(raw)}
    return name, args, str(call.get("id") or default_id or name)


RETRYABLE = {403, 429, 500, 502, 503, 504}


def post_chat(url: str, body: dict, headers: dict | None = None, timeout: int | None = None,
              attempts: int | None = None, log=None, sleep=time.sleep) -> dict:
    """POST one chat completion; retry 403/429/5xx and dropped connections with
    exponential backoff (2, 4, ... 60 s), OCTOPUS_HTTP_ATTEMPTS tries."""
    attempts = attempts or S.http_attempts()
    timeout = timeout or S.http_timeout()
    payload = json.dumps(body).encode()
    delay, last = 2, "request failed"
    for attempt in range(1, attempts + 1):
        req = urllib.request.Request(url, data=payload, headers={"Content-Type": "application/json",
                                                                 **(headers or {})})
        t0 = time.time()
        ev = {"t": t0, "attempt": attempt, "payload_bytes": len(payload)}
        try:
            with urllib.request.urlopen(req, timeout=timeout) as resp:
                raw = resp.read()
                status = getattr(resp, "status", 200)
            data = json.loads(raw.decode())
            usage = data.get("usage") or {}
            ev.update(http_code=status, id=data.get("id"), prompt_tokens=usage.get("prompt_tokens"),
                      completion_tokens=usage.get("completion_tokens"),
                      cached_tokens=(usage.get("prompt_tokens_details") or {}).get("cached_tokens"),
                      elapsed_s=round(time.time() - t0, 3))
            if log:
                log(ev)
            return data
        except urllib.error.HTTPError as exc:
            detail = exc.read().decode("utf-8", "replace")[:300]
            last = f"HTTP {exc.code} {detail}".strip()
            ev.update(http_code=exc.code, error=detail, elapsed_s=round(time.time() - t0, 3))
            if log:
                log(ev)
            if exc.code not in RETRYABLE or attempt == attempts:
                break
        except Exception as exc:  # connection errors, timeouts, bad JSON
            last = f"{type(exc).__name__}: {exc}"
            ev.update(error=last, elapsed_s=round(time.time() - t0, 3))
            if log:
                log(ev)
            if attempt == attempts:
                break
        sleep(delay)
        delay = min(delay * 2, 60)
    raise RuntimeError(last)


# ---------------------------------------------------------------------------- thread names
def branch_ids(owner: str | None, start: int, n: int) -> list[str]:
    """branch-<i> under main (every fork restarts at 0); <owner>.<k> under a branch, numbered on."""
    if owner is None:
        return [f"branch-{i}" for i in range(n)]
    return [f"{owner}.{start + i}" for i in range(n)]


def thread_name(parent: str, k: int, branch_id: str) -> str:
    return f"fork{k}/{branch_id}" if parent == "main" else f"{parent}/fork{k}/{branch_id}"


def branch_key(thread: str) -> str:
    return thread.replace("/", "-")


def tree_branches(forks: list, parent: str = "main"):
    """(thread name, fork record, branch record) for every branch at any depth, depth first."""
    for k, fork in enumerate(forks):
        for br in fork.get("branches") or []:
            name = thread_name(parent, k, br["branch_id"])
            yield name, fork, br
            yield from tree_branches(br.get("forks") or [], name)


# ---------------------------------------------------------------------------- runtime tools
def _tool(name, description, properties, required):
    return {"type": "function", "function": {"name": name, "description": description, "parameters": {
        "type": "object", "additionalProperties": False, "properties": properties, "required": required}}}


FORK_RULE = " A reply whose fork starts cannot also call done, commit or abort: call them in a later reply."
RUNTIME_TOOLS = [
    _tool("fork", "Clone this conversation into N private branches. Need at least two tasks. Each task is that "
                  "branch's next user turn." + FORK_RULE,
          {"tasks": {"type": "array", "items": {"type": "string"}, "minItems": 2}}, ["tasks"]),
    _tool("commit", "Keep one branch's summary for the thread that forked it. Names the branch. Available only after "
                    "a successful fork.",
          {"branch_id": {"type": "string"}, "summary": {"type": "string"}}, ["branch_id", "summary"]),
    _tool("abort", "Drop one branch. The shared prefix stays. Available only after a successful fork.",
          {"branch_id": {"type": "string"}}, ["branch_id"]),
]
DONE_TOOL = _tool("done", "Finish the task with the final answer.", {"answer": {"type": "string"}}, ["answer"])
REWIND_TOOL = _tool(
    "rewind", "Go back to the end of an earlier step of this thread (the step N in each tool result's tag): the "
              "workspace is restored to that step, every later step is removed from your history and your note "
              "stays in their place.",
    {"to_step": {"type": "integer"}, "note": {"type": "string"}}, ["to_step", "note"])
READ_TOOL = _tool(
    "read_thread", "Read another thread of this episode without copying its text: the readable steps from_step to "
                   "to_step are mounted into your attention from your next reply on.",
    {"thread": {"type": "string"}, "from_step": {"type": "integer"}, "to_step": {"type": "integer"}}, ["thread"])
RUNTIME_NAMES = tuple(t["function"]["name"] for t in RUNTIME_TOOLS)
FORK_STARTED = "fork started: branches "
CLOSING = {"done", "commit", "abort"}


def runtime_tools() -> list[dict]:
    tools = list(RUNTIME_TOOLS)
    if S.rewind_tool():
        tools.append(REWIND_TOOL)
    return tools


@dataclass
class RuntimePort:
    """Records one thread's runtime-tool calls and names the branches of its forks (the
    KV cache stays with the engine).  Branches of main are branch-0..n-1 at every fork;
    a branch's own branches are numbered on across its forks (<owner>.<k>)."""

    owner: str | None = None
    forked: int = 0
    calls: list = field(default_factory=list)
    last_fork: dict | None = None

    def fork(self, tasks: list[str]) -> str:
        ids = branch_ids(self.owner, self.forked, len(tasks))
        self.forked += len(ids)
        self.calls.append(("fork", {"tasks": tasks}))
        self.last_fork = {"branches": [{"branch_id": bid, "task": task} for bid, task in zip(ids, tasks)]}
        return FORK_STARTED + ", ".join(ids)

    def commit(self, branch_id: str, summary: str) -> str:
        self.calls.append(("commit", {"branch_id": branch_id, "summary": summary}))
        return f"commit recorded: {branch_id}"

    def abort(self, branch_id: str) -> str:
        self.calls.append(("abort", {"branch_id": branch_id}))
        return f"abort recorded: {branch_id}"


_JSON_ESCAPES = set('"\\/bfnrtu')


def fork_task_list(tasks) -> list | None:
    """A fork's tasks as a list.  Models often send the array as a JSON string with raw
    control characters or stray backslashes: such a string is decoded leniently (control
    characters allowed, a backslash before a non-escape character kept literally, text
    after the array ignored)."""
    if isinstance(tasks, str):
        out, k, text = [], 0, tasks.strip()
        while k < len(text):
            ch = text[k]
            if ch == "\\" and k + 1 < len(text):
                nxt = text[k + 1]
                out.append(ch + nxt if nxt in _JSON_ESCAPES else "\\\\" + nxt)
                k += 2
                continue
            out.append(ch)
            k += 1
        tasks, _ = json.JSONDecoder(strict=False).raw_decode("".join(out))
    return tasks if isinstance(tasks, list) else None


def _text_arg(args: dict, key: str) -> str | None:
    v = args.get(key)
    return v if isinstance(v, str) and v.strip() else None


def _fork(args: dict, port: RuntimePort, need: str, fewest: int) -> str:
    try:
        tasks = fork_task_list(args.get("tasks"))
    except json.JSONDecodeError as e:
        return (f"fork refused: tasks is not a JSON array ({e.msg} at char {e.pos}). Send [\"...\", ...]; "
                "escape every \" inside a string.")
    valid = tasks is not None and len(tasks) >= max(1, fewest) and all(
        isinstance(x, str) and x.strip() for x in tasks)
    if not valid:
        return f"fork needs at least two {need}" if fewest > 1 else f"fork needs {need}"
    return port.fork(list(tasks))


def apply_runtime(name: str, args: dict | None, port: RuntimePort | None = None, need: str = "tasks",
                  needs=None, fewest: int = 2) -> tuple[str, bool]:
    """Validate and record one runtime-tool call; returns (observation, stop=False).
    `needs(name, args)` may veto a commit / abort with a message (a gate)."""
    port = port if port is not None else RuntimePort()
    args = dict(args or {})
    if name == "fork":
        return _fork(args, port, need, fewest), False
    if name not in ("commit", "abort"):
        return f"unknown runtime tool {name}", False
    bid = _text_arg(args, "branch_id")
    if name == "commit":
        summary = _text_arg(args, "summary")
        if bid is None or summary is None:
            return "commit needs branch_id and summary", False
    elif bid is None:
        return "abort needs branch_id", False
    veto = needs(name, args) if needs else None
    if veto:
        return veto, False
    return (port.commit(bid, args["summary"]) if name == "commit" else port.abort(bid)), False


def rejected(name: str | None, observed) -> bool:
    return name in ("commit", "abort") and str(observed or "").startswith(("commit needs", "abort needs"))


def started(name: str, observed) -> bool:
    return name == "fork" and str(observed).startswith(FORK_STARTED)


def _accepted(steps: list[dict]):
    return (s for s in reversed(steps) if s.get("name") and not s.get("rejected"))


def closing_step(steps: list[dict]) -> dict | None:
    """The thread's last accepted closing call (done / commit / abort), if any."""
    return next((s for s in _accepted(steps) if s["name"] in CLOSING), None)


def handed(closing: dict | None) -> str | None:
    a = (closing or {}).get("arguments") or {}
    return a.get("summary", a.get("answer"))


def closing_name(steps: list[dict]) -> str | None:
    last = next(_accepted(steps), None)
    return last["name"] if last else None


def add_note(messages: list, text: str, pending: bool = True) -> None:
    """Append a runtime note.  It is a user message, except in thinking mode, where it
    joins the tool results just sent (or becomes a tool message of its own)."""
    if pending and not S.thinking():
        messages.append({"role": "user", "content": text})
        return
    if pending and messages and messages[-1].get("role") == "tool":
        messages[-1] = {**messages[-1], "content": f"{messages[-1]['content']}\n\n{text}"}
        return
    messages.append({"role": "tool", "content": text})


# Model-visible notes (the wording is part of the runtime's interface with the policy).
RESERVE_NOTE = ("Refused: your context is nearly used up ({left} tokens left). Close now: call {calls} with what you "
                "have so far{rewind}. Until you do, every other call is refused.")
CLIPPED = "[clipped: context nearly used up]"
CLOSE_NOTE = ("Your context is nearly used up. Close now: call {calls} with what you have so far{rewind}; any other "
              "call is refused.")
REWIND_FREES = ", or rewind to an earlier step to free context"
REMIND_NOTE = ("You replied without a tool call. A thread's result counts only through its closing call: close with "
               "{calls} now, or continue with a tool call.")
REWIND_SPENT = "No rewinds left (at most {} per thread); nothing was rewound."
FORK_ALONE = "{0} refused: a reply whose fork started cannot also call {0}. Call it in a later reply."
MESSAGE_TOKENS = 40  # framing tokens per tool message, counted against the room


_TOKENIZERS: dict = {}


def count_tokens(text: str) -> int:
    """Tokens of `text` under the policy's tokenizer (OCTOPUS_TOKENIZER: a folder with
    tokenizer.json), else an estimate of one token per 4 characters."""
    path = os.environ.get("OCTOPUS_TOKENIZER")
    if not path:
        return (len(text) + 3) // 4
    if path not in _TOKENIZERS:
        from tokenizers import Tokenizer

        _TOKENIZERS[path] = Tokenizer.from_file(os.path.join(path, "tokenizer.json"))
    return len(_TOKENIZERS[path].encode(text, add_special_tokens=False).ids)


def _longest_prefix(text: str, tokens: int) -> int:
    """Largest n such that text[:n] takes at most `tokens` tokens (token counts grow with
    the prefix, so a bisection over n finds it)."""
    return bisect.bisect_right(range(len(text) + 1), tokens, key=lambda n: count_tokens(text[:n])) - 1


def clip_results(results: list[str], room: int, note: str) -> list[str] | None:
    """Tool results cut to fit `room` tokens, or None when they already fit.  Results are
    kept in order while they fit; the first that does not, and every later one, is cut to
    what is left (possibly nothing) and marked CLIPPED; `note` ends the last result."""
    sizes = [count_tokens(r) for r in results]
    budget = room - MESSAGE_TOKENS * len(results)
    if sum(sizes) <= budget:
        return None
    budget -= count_tokens("\n\n" + note) + len(results) * count_tokens("\n" + CLIPPED)
    out, spent = [], 0
    for text, size in zip(results, sizes):
        free = max(0, budget - spent)
        out.append(text if size <= free else text[:_longest_prefix(text, free)] + "\n" + CLIPPED)
        spent += size
    out[-1] = out[-1] + "\n\n" + note
    return out


def step_number(raw) -> int | None:
    if isinstance(raw, bool):
        return None
    if isinstance(raw, int):
        return raw
    if isinstance(raw, str) and raw.strip().isdigit():
        return int(raw)
    return None


async def _maybe(x):
    return await x if hasattr(x, "__await__") else x


class _Context:
    """A thread's context accounting: prompt growth since its first request against the
    growth budget (tightened to the model's window room), the answer reserve, and whether
    results were already clipped."""

    def __init__(self, budget: int | None, mounted: int):
        self.budget = budget
        self.reserve = S.answer_reserve() if budget else 0
        self.mounted = mounted
        self.first: int | None = None
        self.grown = 0
        self.clipped = False

    def left(self) -> int:
        return max(0, self.budget - self.grown) if self.budget else 0

    def observe(self, usage: dict) -> str | None:
        """Account one response; returns a stop message if the prompt outgrew the budget."""
        prompt = usage.get("prompt_tokens")
        if self.first is None and prompt:
            self.first = prompt
        if self.budget and prompt and prompt - self.first > self.budget:
            return f"stopped: grew {prompt - self.first} tokens past its start (budget {self.budget})"
        if prompt:
            self.grown = prompt - self.first + int(usage.get("completion_tokens") or 0)
        return None

    def tighten(self):
        if self.budget and self.first:
            self.budget = max(1, min(self.budget, S.window_room(self.first + self.mounted)))

    def in_reserve(self) -> bool:
        return self.clipped or bool(self.reserve and self.budget - self.grown < self.reserve)

    def exhausted(self) -> bool:
        return bool(self.budget and self.budget - self.grown < max(self.reserve, 1))

    def rewound_to(self, prompt: int | None):
        if prompt and self.first:
            self.grown = prompt - self.first
        self.clipped = self.clipped and self.budget - self.grown < self.reserve


@dataclass
class _Mark:
    """End of one step of the thread: message count, step-record count, the prompt size
    seen at it, and a workspace snapshot taken before the step's first working call."""

    end: int
    steps: int
    snap: object = None
    prompt: int | None = None


@dataclass
class _Call:
    name: str
    args: dict
    cid: str
    observed: str = ""
    stop: bool = False
    refused: bool = False
    fields: dict = field(default_factory=dict)


class _ThreadLoop:
    """One thread's turns until it closes; run_thread documents the contract."""

    def __init__(self, start, complete, dispatch, max_steps, closing, budget, join, refused, max_calls, before_turn,
                 snapshot, restore, log, ws):
        self.start, self.complete, self.dispatch = start, complete, dispatch
        self.max_steps, self.max_calls, self.closing = max_steps, max_calls, set(closing)
        self.join, self.refused, self.before_turn = join, refused, before_turn
        self.snapshot, self.restore, self.ws = snapshot, restore, ws
        self.log = log or (lambda kind, **f: None)
        self.messages = start["messages"]
        self.sid, self.bid = start["session_id"], start["branch_id"]
        self.base = start.get("step") or 0
        start["reminded"] = start.get("reminded") or 0
        start.setdefault("rewinds_used", 0)
        self.ctx = _Context(budget, start.get("mounted", 0))
        self.marks = [_Mark(len(self.messages), 0)]
        self.steps: list[dict] = []
        self.rewinds: list[dict] = []
        self.turns = self.calls = 0
        self.rewind_on, self.rewind_cap = S.rewind_tool(), S.rewind_max()
        self.notes = {"calls": " or ".join(sorted(self.closing)), "rewind": ""}

    # ------------------------------------------------------------------ helpers
    @property
    def current_step(self) -> int:
        return self.base + len(self.marks) - 1

    def _end(self, text: str):
        self.steps.append({"name": None, "text": text, "session_id": self.sid, "arguments": {}})
        self.log("end", text=text)

    def _may_continue(self) -> bool:
        return ((self.max_steps is None or self.turns < self.max_steps)
                and (self.max_calls is None or self.calls < self.max_calls))

    def _publish_limits(self):
        left = [cap - used for cap, used in ((self.max_steps, self.turns), (self.max_calls, self.calls))
                if cap is not None]
        self.start["calls_left"] = min(left) if left else None
        if self.ctx.budget:
            self.start["context_left"] = self.ctx.left()
        self.start["step"] = self.current_step

    def _rewinds_spent(self) -> bool:
        return bool(self.rewind_cap) and self.start["rewinds_used"] >= self.rewind_cap

    def _push_mark(self):
        self.marks.append(_Mark(len(self.messages), len(self.steps)))

    # ------------------------------------------------------------------ one call
    async def _run_call(self, call: _Call, reserved: bool, fork_started: bool) -> tuple[_Call, tuple | None]:
        """Execute (or refuse) one call; returns it and a pending rewind target, if any."""
        is_rewind = self.rewind_on and call.name == "rewind"
        if fork_started and (call.name in self.closing or is_rewind):
            call.observed, call.refused = FORK_ALONE.format(call.name), True
            call.fields["alone"] = True
            return call, None
        if reserved and call.name not in self.closing and not is_rewind:
            call.observed = RESERVE_NOTE.format(left=self.ctx.left(), **self.notes)
            call.refused = True
            return call, None
        if self.rewind_on and self.snapshot and self.marks[-1].snap is None and call.name not in ("rewind",
                                                                                                  "read_thread"):
            self.marks[-1].snap = await _maybe(self.snapshot())
        if is_rewind:
            return self._rewind_call(call)
        if self.ws is not None and call.name == "commit" and "commit" in self.closing:
            gate, extra = await self.ws.check_close(self.start, call.args, True, None)
            if gate:
                call.observed, call.refused = gate, True
                call.fields.update(gated=True, **extra)
                return call, None
            call.fields.update(extra)
        call.observed, call.stop = await _maybe(self.dispatch(call.name, call.args, self.bid))
        call.refused = bool(self.refused(call.name, call.observed)) or (
            call.name in CLOSING and call.name not in self.closing)
        return call, None

    def _rewind_call(self, call: _Call) -> tuple[_Call, tuple | None]:
        if self._rewinds_spent():
            call.observed, call.refused = REWIND_SPENT.format(self.rewind_cap), True
            return call, None
        to = step_number(call.args.get("to_step"))
        if to is None or not self.base <= to <= self.current_step:
            call.observed = (f"rewind needs to_step, one of this thread's steps: an integer from {self.base} to "
                             f"{self.current_step}. Nothing was rewound.")
            return call, None
        call.observed = f"rewound to step {to}"
        return call, (to, call.args.get("note") or "", len(self.steps))

    def _record(self, call: _Call):
        rec = {"name": call.name, "arguments": call.args, "tool_call_id": call.cid, "session_id": self.sid,
               "branch_id": self.bid, "observed": call.observed}
        if call.refused:
            rec["rejected"] = True
        rec.update({k: v for k, v in call.fields.items() if k != "alone"})
        self.steps.append(rec)

    # ------------------------------------------------------------------ rewind
    async def _apply_rewind(self, target: tuple):
        to, note, _ = target
        mark = self.marks[to - self.base]
        if self.restore and mark.snap is not None:
            await _maybe(self.restore(mark.snap))
        dropped = self.messages[mark.end:]
        self.rewinds.append({"step": len(self.steps), "to_step": to, "dropped_messages": len(dropped),
                             "messages": dropped, "note": note})
        del self.messages[mark.end:]
        add_note(self.messages, f"[rewound to step {to}] {note}", pending=False)
        del self.marks[to - self.base + 1:]
        self.marks[-1] = _Mark(len(self.messages), len(self.steps), mark.snap, mark.prompt)
        self.ctx.rewound_to(mark.prompt)
        self.start["rewinds_used"] += 1
        self.log("rewind", **self.rewinds[-1])

    # ------------------------------------------------------------------ turns
    async def _reply_without_calls(self, payload: dict, choice: dict, text: str) -> bool:
        """Remind once; returns False when the thread ends here."""
        self.ctx.tighten()
        room = ((self.max_steps is None or self.turns < self.max_steps) and not self.ctx.clipped
                and not self.ctx.exhausted() and not payload.get("budget_out"))
        if self.start["reminded"] or not room:
            self._end(text)
            return False
        self.start["reminded"] += 1
        self.messages.append(with_cursor(reply_message(choice, text), payload))
        add_note(self.messages, REMIND_NOTE.format(**self.notes))
        self._push_mark()
        self.log("remind", text=text)
        return True

    async def _turn(self) -> bool:
        """One request and its calls; returns False when the thread ends."""
        stop_why = self.before_turn(self.turns) if self.before_turn else None
        if stop_why:
            self._end(f"stopped: {stop_why}")
            return False
        self._publish_limits()
        self.turns += 1
        try:
            payload = await _maybe(self.complete(self.messages, self.sid))
        except Exception as exc:
            self._end(f"request failed: {exc}")
            return False
        usage = payload.get("usage") or {}
        if usage.get("prompt_tokens"):
            self.marks[-1].prompt = usage["prompt_tokens"]
        overflow = self.ctx.observe(usage)
        if overflow:
            self.steps.append({"name": "context", "arguments": {}, "session_id": self.sid, "observed": overflow})
            return False
        reserved = self.ctx.in_reserve()
        self.notes["rewind"] = REWIND_FREES if self.rewind_on and not self._rewinds_spent() else ""
        choice = (payload.get("choices") or [{}])[0].get("message") or {}
        raw_calls, text = reply_tools(choice)
        if not raw_calls:
            return await self._reply_without_calls(payload, choice, text)

        done: list[_Call] = []
        target, fork_started, closed = None, False, False
        for idx, raw in enumerate(raw_calls):
            name, args, cid = decode_tool_call(raw, default_id=f"{self.bid}-{len(self.steps)}-{idx}")
            call, pending = await self._run_call(_Call(name, args, cid), reserved, fork_started)
            target = pending or target
            self._record(call)
            done.append(call)
            fork_started = fork_started or started(call.name, call.observed)
            if call.stop or (call.name in self.closing and not call.refused):
                closed = True
                break
        if target is not None and fork_started:  # a rewind in the reply that forked is refused
            step = self.steps[target[2]]
            step.update(observed=FORK_ALONE.format("rewind"), rejected=True)
            done[target[2] - (len(self.steps) - len(done))].observed = step["observed"]
            done[target[2] - (len(self.steps) - len(done))].fields["alone"] = True
            target = None
        self.ctx.tighten()
        observations = [c.observed for c in done]
        if self.ctx.reserve and not reserved and not closed and target is None:
            cut = clip_results([str(o) for o in observations],
                               self.ctx.budget - self.ctx.reserve - self.ctx.grown, CLOSE_NOTE.format(**self.notes))
            if cut:
                observations = cut
                self.ctx.clipped = True
        self.messages.append(with_cursor(reply_message(choice, text, raw_calls[:len(done)]), payload))
        self.messages.extend({"role": "tool", "tool_call_id": c.cid, "content": o} for c, o in zip(done, observations))
        self.calls += sum(1 for c in done if not c.fields.get("alone"))
        for c, o in zip(done, observations):
            self.log("call", name=c.name, args=c.args, call_id=c.cid, observed=o, text=text)
        note = await self.join(self.messages) if self.join else None
        if note:
            add_note(self.messages, note)
        self._push_mark()
        if target is not None and not closed:
            await self._apply_rewind(target)
        return not closed

    async def run(self) -> dict:
        while self._may_continue():
            if not await self._turn():
                break
        return {"rewinds": self.rewinds, "reminded": self.start["reminded"], "branch_id": self.bid,
                "session_id": self.sid, "task": self.start.get("task"), "steps": self.steps,
                "messages": self.messages}


async def run_thread(start: dict, complete, dispatch, max_steps: int | None = 8, closing=CLOSING,
                     budget: int | None = None, join=None, *, refused=rejected, max_calls: int | None = None,
                     before_turn=None, snapshot=None, restore=None, log=None, ws=None) -> dict:
    """Run one thread until it closes.

    start: {branch_id, session_id, task, messages, [step, mounted, reminded]}; the loop
    writes calls_left / context_left / step into it before each request.
    complete(messages, session_id) -> chat payload (OpenAI shape; may be a coroutine).
    dispatch(name, args, branch_id) -> (observation, stop) for every non-rewind call.
    join(messages) -> a note to append after each turn's tool results, or None.

    Rules: at most max_steps requests and max_calls counted calls; a reply without a tool
    call gets one reminder, then ends the thread; a reply whose fork started cannot also
    close or rewind; once the answer reserve is reached (or results were clipped) only
    closing calls and rewinds run; results that would cross the reserve are clipped with
    a close note; the rewind tool restores the workspace snapshot of the target step and
    cuts the history back to it (at most OCTOPUS_REWIND_MAX per thread); a closing call
    (done / commit / abort, as allowed for the thread) that is accepted ends the thread.
    """
    loop = _ThreadLoop(start, complete, dispatch, max_steps, closing, budget, join, refused, max_calls, before_turn,
                       snapshot, restore, log, ws)
    return await loop.run()


run_branch_continuation = run_thread  # the reference's name for the same loop


# ---------------------------------------------------------------------------- fork / join text
BRANCH_REPORT = "findings, files, changes"


def branch_task_message(branch_id: str, task: str, siblings: int, report: str = BRANCH_REPORT,
                        contract: str | None = None, close: str = "") -> str:
    who = (f"You are {branch_id}, one of {siblings} parallel branches cloned from the context above.\n"
           if siblings > 1 else f"You are {branch_id}, the one branch cloned from the context above.\n")
    how = contract if contract is not None else (
        f'When it is done, call commit with branch_id="{branch_id}" and a summary the thread that forked you can act '
        f'on ({report}). If it cannot be done, call abort with branch_id="{branch_id}".')
    return who + f"Your task: {task}\nWork only on this task. " + how + (" " + close if close else "")


def join_note(results: list[dict]) -> str:
    """What the forking thread is told when its branches are collected."""
    lines = []
    for r in results:
        how = r.get("ended_with") or "ended"
        summ = r.get("summary")
        lines.append(f"- {r['branch_id']}: {how}" + (f": {summ}" if summ else ""))
    return "Branches finished:\n" + "\n".join(lines)


def fork_record(port: RuntimePort, response_id: str | None, history_len: int) -> dict:
    return {"response_id": response_id, "history_len": history_len,
            "branches": [dict(b) for b in (port.last_fork or {}).get("branches", [])]}


def token_counts(requests: list[dict]) -> dict:
    c = collections.Counter()
    for r in requests:
        c["prompt"] += int(r.get("prompt_tokens") or 0)
        c["completion"] += int(r.get("completion_tokens") or 0)
        c["cached"] += int(r.get("cached_tokens") or 0)
    return dict(c)
