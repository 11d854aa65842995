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
    """(cursor of the last reply carrying one, the messages after it); (None, all) if none."""
    for i in range(len(messages) - 1, -1, -1):
        if "cursor" in messages[i]:
            return messages[i]["cursor"], messages[i + 1:]
    return None, messages


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


class RuntimePort:
    """Records runtime tool calls and assigns branch ids (KV stays the engine's)."""

    def __init__(self, owner: str | None = None):
        self.owner = owner
        self.forked = 0
        self.calls: list[tuple[str, dict]] = []
        self.last_fork: dict | None = None

    def fork(self, tasks: list[str]) -> str:
        self.calls.append(("fork", {"tasks": tasks}))
        ids = branch_ids(self.owner, self.forked, len(tasks))
        self.forked += len(tasks)
        self.last_fork = {"branches": [{"branch_id": b, "task": t} for b, t in zip(ids, tasks)]}
        return FORK_STARTED + ", ".join(ids)

    def commit(self, branch_id: str, summary: str) -> str:
        self.calls.append(("commit", {"branch_id": branch_id, "summary": summary}))
        return f"commit recorded: {branch_id}"

    def abort(self, branch_id: str) -> str:
        self.calls.append(("abort", {"branch_id": branch_id}))
        return f"abort recorded: {branch_id}"


def fork_task_list(tasks) -> list | None:
    """A fork's tasks as a list: a JSON string is parsed leniently (raw control characters
    inside strings, stray backslashes kept, trailing text ignored)."""
    if isinstance(tasks, str):
        text = tasks.strip()
        fixed = re.sub(r"\\(.)", lambda m: m[0] if m[1] in '"\\/bfnrtu' else "\\" + m[0], text, flags=re.S)
        tasks = json.JSONDecoder(strict=False).raw_decode(fixed)[0]
    return tasks if isinstance(tasks, list) else None


def apply_runtime(name: str, args: dict | None, port: RuntimePort | None = None, need: str = "tasks",
                  needs=None, fewest: int = 2) -> tuple[str, bool]:
    port = port or RuntimePort()
    args = dict(args or {})
    if name == "fork":
        try:
            tasks = fork_task_list(args.get("tasks"))
        except json.JSONDecodeError as e:
            return (f"fork refused: tasks is not a JSON array ({e.msg} at char {e.pos}). Send [\"...\", ...]; "
                    "escape every \" inside a string."), False
        tasks = [t if isinstance(t, str) and t.strip() else None for t in tasks] if isinstance(tasks, list) else None
        if not tasks or len(tasks) < fewest or any(t is None for t in tasks):
            return (f"fork needs at least two {need}" if fewest > 1 else f"fork needs {need}"), False
        return port.fork(list(tasks)), False
    if name == "commit":
        bid, summ = args.get("branch_id"), args.get("summary")
        if not isinstance(bid, str) or not bid.strip() or not isinstance(summ, str) or not summ.strip():
            return "commit needs branch_id and summary", False
        lack = needs and needs(name, args)
        return (lack, False) if lack else (port.commit(bid, summ), False)
    if name == "abort":
        bid = args.get("branch_id")
        if not isinstance(bid, str) or not bid.strip():
            return "abort needs branch_id", False
        lack = needs and needs(name, args)
        return (lack, False) if lack else (port.abort(bid), False)
    return f"unknown runtime tool {name}", False


def rejected(name: str | None, observed) -> bool:
    return name in {"commit", "abort"} and str(observed or "").startswith(("commit needs", "abort needs"))


def started(name: str, observed) -> bool:
    return name == "fork" and str(observed).startswith(FORK_STARTED)


def closing_step(steps: list[dict]) -> dict | None:
    return next((s for s in reversed(steps) if s.get("name") in CLOSING and not s.get("rejected")), None)


def handed(closing: dict | None) -> str | None:
    a = (closing or {}).get("arguments") or {}
    return a.get("summary", a.get("answer"))


def closing_name(steps: list[dict]) -> str | None:
    return next((s["name"] for s in reversed(steps) if s.get("name") and not s.get("rejected")), None)


def add_note(messages: list, text: str, pending: bool = True) -> None:
    """A runtime note: a user message, or (thinking mode / after sent results) a tool message."""
    if pending and not S.thinking():
        messages.append({"role": "user", "content": text})
    elif pending and messages and messages[-1].get("role") == "tool":
        messages[-1] = dict(messages[-1], content=f"{messages[-1]['content']}\n\n{text}")
    else:
        messages.append({"role": "tool", "content": text})


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
MESSAGE_TOKENS = 40


def count_tokens(text: str) -> int:
    """Tokens of `text` under the policy tokenizer (OCTOPUS_TOKENIZER) or a 4-char estimate."""
    path = os.environ.get("OCTOPUS_TOKENIZER")
    if path:
        from tokenizers import Tokenizer
        tok = _TOKENIZERS.get(path)
        if tok is None:
            tok = _TOKENIZERS.setdefault(path, Tokenizer.from_file(os.path.join(path, "tokenizer.json")))
        return len(tok.encode(text, add_special_tokens=False).ids)
    return (len(text) + 3) // 4


_TOKENIZERS: dict = {}


def clip_results(results: list[str], room: int, note: str) -> list[str] | None:
    """Cut tool results to `room` tokens (binary search on the character cut), each cut one
    ending with CLIPPED and the last with `note`; None when they fit."""
    sizes = [count_tokens(t) for t in results]
    left = room - MESSAGE_TOKENS * len(results)
    if sum(sizes) <= left:
        return None
    left -= count_tokens("\n\n" + note) + count_tokens("\n" + CLIPPED) * len(results)
    out = []
    for text, size in zip(results, sizes):
        keep = max(0, left)
        if size <= keep:
            out.append(text)
        else:
            lo, hi = 0, len(text)
            while lo < hi:
                mid = (lo + hi + 1) // 2
                if count_tokens(text[:mid]) <= keep:
                    lo = mid
                else:
                    hi = mid - 1
            out.append(text[:lo] + "\n" + CLIPPED)
        left -= size
    out[-1] += "\n\n" + note
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


async def run_thread(start: dict, complete, dispatch, max_steps: int | None = 8, closing=CLOSING,
                     budget: int | None = None, join=None, *, refused=rejected, max_calls: int | None = None,
                     before_turn=None, snapshot=None, restore=None, log=None, ws=None) -> dict:
    """Run one thread until it closes (see module docstring for the rules).

    start: {branch_id, session_id, task, messages, [step, mounted, reminded]}.
    complete(messages, session_id) -> chat payload (OpenAI shape, may be async).
    dispatch(name, args, branch_id) -> (observation, stop) for working tools.
    join(messages) -> note or None, awaited after each turn's tool results.
    """
    messages = start["messages"]
    sid, bid = start["session_id"], start["branch_id"]
    steps: list[dict] = []
    first_prompt, grown = None, 0
    base = start.get("step") or 0
    marks = [{"end": len(messages), "steps": 0, "snap": None}]
    start["reminded"] = start.get("reminded") or 0
    start.setdefault("rewinds_used", 0)
    turns = calls = 0
    reserve = S.answer_reserve() if budget else 0
    clipped = False
    tool_rewind, cap = S.rewind_tool(), S.rewind_max()
    rewinds: list[dict] = []
    allowed = {"calls": " or ".join(sorted(closing))}
    log = log or (lambda kind, **f: None)

    def end(text):
        steps.append({"name": None, "text": text, "session_id": sid, "arguments": {}})
        log("end", text=text)

    while (max_steps is None or turns < max_steps) and (max_calls is None or calls < max_calls):
        reason = before_turn(turns) if before_turn else None
        if reason:
            end(f"stopped: {reason}")
            break
        left = [c - u for c, u in ((max_steps, turns), (max_calls, calls)) if c is not None]
        start["calls_left"] = min(left) if left else None
        if budget:
            start["context_left"] = max(0, budget - grown)
        start["step"] = base + len(marks) - 1
        turns += 1
        try:
            payload = await _maybe(complete(messages, sid))
        except Exception as exc:
            end(f"request failed: {exc}")
            break
        usage = payload.get("usage") or {}
        prompt = usage.get("prompt_tokens")
        first_prompt = first_prompt or prompt
        if prompt:
            marks[-1]["prompt"] = prompt
        if budget and prompt and first_prompt and prompt - first_prompt > budget:
            steps.append({"name": "context", "arguments": {}, "session_id": sid,
                          "observed": f"stopped: grew {prompt - first_prompt} tokens past its start (budget {budget})"})
            break
        if prompt and first_prompt:
            grown = prompt - first_prompt + int(usage.get("completion_tokens") or 0)
        reserved = clipped or (reserve and budget - grown < reserve)
        spent = cap and start["rewinds_used"] >= cap
        allowed["rewind"] = REWIND_FREES if tool_rewind and not spent else ""
        choice = (payload.get("choices") or [{}])[0].get("message") or {}
        calls_in, text = reply_tools(choice)
        if not calls_in:
            if budget and first_prompt:
                budget = max(1, min(budget, S.window_room(first_prompt + start.get("mounted", 0))))
            room = ((max_steps is None or turns < max_steps) and not clipped
                    and not (budget and budget - grown < max(reserve, 1)) and not payload.get("budget_out"))
            if start["reminded"] or not room:
                end(text)
                break
            start["reminded"] += 1
            messages.append(with_cursor(reply_message(choice, text), payload))
            add_note(messages, REMIND_NOTE.format(**allowed))
            marks.append({"end": len(messages), "steps": len(steps), "snap": None})
            log("remind", text=text)
            continue
        stop, executed, back, forked, alone_n = False, [], None, False, 0
        for idx, call in enumerate(calls_in):
            name, args, cid = decode_tool_call(call, default_id=f"{bid}-{len(steps)}-{idx}")
            alone = forked and (name in closing or (tool_rewind and name == "rewind"))
            held = (reserved and name not in closing and not (tool_rewind and name == "rewind")) or alone
            if tool_rewind and snapshot and marks[-1]["snap"] is None and not held and name not in ("rewind",
                                                                                                 "read_thread"):
                marks[-1]["snap"] = await _maybe(snapshot())
            fields = {}
            if alone:
                observed, cstop, refusal = FORK_ALONE.format(name), False, True
                alone_n += 1
            elif held:
                observed, cstop, refusal = RESERVE_NOTE.format(left=max(0, budget - grown), **allowed), False, True
            elif tool_rewind and name == "rewind":
                to = step_number(args.get("to_step"))
                last_step = base + len(marks) - 1
                if spent:
                    observed, cstop, refusal = REWIND_SPENT.format(cap), False, True
                elif to is None or not base <= to <= last_step:
                    observed = (f"rewind needs to_step, one of this thread's steps: an integer from {base} to "
                                f"{last_step}. Nothing was rewound.")
                    cstop, refusal = False, False
                else:
                    back = (to, args.get("note") or "", len(steps))
                    observed, cstop, refusal = f"rewound to step {to}", False, False
            else:
                if ws is not None and name == "commit" and name in closing:
                    gate, fields = await ws.check_close(start, args, True, None)
                    if gate:
                        observed, cstop, refusal = gate, False, True
                        steps.append({"name": name, "arguments": args, "tool_call_id": cid, "session_id": sid,
                                      "branch_id": bid, "observed": observed, "rejected": True, "gated": True,
                                      **fields})
                        executed.append((name, args, cid, observed))
                        continue
                observed, cstop = await _maybe(dispatch(name, args, bid))
                refusal = refused(name, observed) or (name in CLOSING and name not in closing)
            steps.append({"name": name, "arguments": args, "tool_call_id": cid, "session_id": sid, "branch_id": bid,
                          "observed": observed, **({"rejected": True} if refusal else {}), **fields})
            executed.append((name, args, cid, observed))
            forked = forked or started(name, observed)
            if cstop or (name in closing and not refusal):
                stop = True
                break
        if back and forked:
            i = back[2]
            steps[i].update(observed=FORK_ALONE.format("rewind"), rejected=True)
            back = None
            alone_n += 1
        if budget and first_prompt:
            budget = max(1, min(budget, S.window_room(first_prompt + start.get("mounted", 0))))
        if reserve and not reserved and not stop and not back:
            cut = clip_results([str(o) for *_, o in executed], budget - reserve - grown,
                               CLOSE_NOTE.format(**allowed))
            if cut:
                executed = [(*e[:3], o) for e, o in zip(executed, cut)]
                clipped = True
        messages.append(with_cursor(reply_message(choice, text, calls_in[:len(executed)]), payload))
        messages += [{"role": "tool", "tool_call_id": cid, "content": o} for _, _, cid, o in executed]
        calls += len(executed) - alone_n
        for name, args, cid, o in executed:
            log("call", name=name, args=args, call_id=cid, observed=o, text=text)
        note = await join(messages) if join else None
        if note:
            add_note(messages, note)
        marks.append({"end": len(messages), "steps": len(steps), "snap": None})
        if back and not stop:
            to, note_text, _ = back
            mark = marks[to - base]
            if restore and mark.get("snap") is not None:
                await _maybe(restore(mark["snap"]))
            rewinds.append({"step": len(steps), "to_step": to, "dropped_messages": len(messages) - mark["end"],
                            "messages": messages[mark["end"]:], "note": note_text})
            del messages[mark["end"]:]
            add_note(messages, f"[rewound to step {to}] {note_text}", pending=False)
            del marks[to - base + 1:]
            marks[-1] = dict(mark, end=len(messages), steps=len(steps))
            if mark.get("prompt") and first_prompt:
                grown = mark["prompt"] - first_prompt
            clipped = clipped and budget - grown < reserve
            start["rewinds_used"] += 1
            log("rewind", **rewinds[-1])
        if stop:
            break
    return {"rewinds": rewinds, "reminded": start["reminded"], "branch_id": bid, "session_id": sid,
            "task": start.get("task"), "steps": steps, "messages": messages}


# the reference's name for the same loop
run_branch_continuation = run_thread


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
