"""The thread loop's context rules on scripted replies: the answer reserve refuses working
calls, results that would cross it are clipped with the close note, the rewind tool cuts
the history back to a step and restores its snapshot, a rewind in the reply that forked
is refused, and the result clipper keeps results whole while they fit."""
import asyncio
import json

from octopus_b200.runtime import core


def _reply(calls, prompt, completion=10, text=""):
    tc = [{"id": f"c{i}", "type": "function", "function": {"name": n, "arguments": json.dumps(a)}}
          for i, (n, a) in enumerate(calls)]
    return {"choices": [{"message": {"role": "assistant", "content": text, "tool_calls": tc or None}}],
            "usage": {"prompt_tokens": prompt, "completion_tokens": completion}}


def _run(replies, dispatch, **kw):
    it = iter(replies)
    start = {"branch_id": "main", "session_id": "s", "task": "t", "messages": [{"role": "user", "content": "go"}]}
    return asyncio.run(core.run_thread(start, lambda m, sid: next(it), dispatch, **kw))


def test_clip_results_keeps_whole_results_while_they_fit():
    assert core.clip_results(["a" * 40, "b" * 40], 1000, "close") is None
    out = core.clip_results(["a" * 400, "b" * 4000], 40 * 2 + 300, "close now")
    assert out[0] == "a" * 400  # 100 tokens fit
    assert out[1].startswith("b") and core.CLIPPED in out[1] and out[1].endswith("close now")
    assert core.count_tokens(out[1]) < 400


def test_reserve_refuses_working_calls_and_clips(monkeypatch):
    monkeypatch.setenv("OCTOPUS_ANSWER_RESERVE", "200")
    seen = []

    def dispatch(name, args, bid):
        seen.append(name)
        if name == "done":
            return "finished", True
        return "x" * 4000, False  # ~1000 tokens: crosses the reserve

    replies = [_reply([("shell", {"cmd": "ls"})], prompt=1000),
               _reply([("shell", {"cmd": "ls"})], prompt=1900),          # clipped before: only closing calls
               _reply([("done", {"answer": "ok"})], prompt=2000)]
    res = _run(replies, dispatch, budget=1000, max_steps=5)
    msgs = res["messages"]
    first_result = next(m for m in msgs if m.get("role") == "tool")
    assert core.CLIPPED in first_result["content"] and "Close now" in first_result["content"]
    steps = res["steps"]
    assert steps[1]["name"] == "shell" and steps[1].get("rejected") and steps[1]["observed"].startswith("Refused")
    assert seen == ["shell", "done"] and steps[-1]["name"] == "done"


def test_rewind_cuts_history_and_restores_snapshot(monkeypatch):
    monkeypatch.setenv("OCTOPUS_REWIND_TOOL", "1")
    state = {"ws": 0, "restored": None}

    def dispatch(name, args, bid):
        if name == "done":
            return "finished", True
        state["ws"] += 1
        return f"edit {state['ws']}", False

    async def snapshot():
        return state["ws"]

    async def restore(snap):
        state["restored"] = snap
        state["ws"] = snap

    replies = [_reply([("edit", {"path": "a"})], prompt=100),       # step 0
               _reply([("edit", {"path": "b"})], prompt=200),       # step 1
               _reply([("rewind", {"to_step": 1, "note": "undo b"})], prompt=300),
               _reply([("done", {"answer": "ok"})], prompt=150)]
    res = _run(replies, dispatch, snapshot=snapshot, restore=restore, max_steps=10)
    assert state["restored"] == 1 and state["ws"] == 1  # workspace back to the end of step 0
    assert len(res["rewinds"]) == 1 and res["rewinds"][0]["to_step"] == 1
    contents = [str(m.get("content")) for m in res["messages"]]
    assert any(c.startswith("[rewound to step 1] undo b") for c in contents)
    assert not any(c == "edit 2" for c in contents)  # step 1's result was cut from the history


def test_rewind_in_the_forking_reply_is_refused(monkeypatch):
    monkeypatch.setenv("OCTOPUS_REWIND_TOOL", "1")

    def dispatch(name, args, bid):
        if name == "fork":
            return core.FORK_STARTED + "branch-0, branch-1", False
        if name == "done":
            return "finished", True
        return "ok", False

    replies = [_reply([("edit", {"path": "a"})], prompt=100),
               _reply([("rewind", {"to_step": 0, "note": "n"}), ("fork", {"tasks": ["a", "b"]})], prompt=200),
               _reply([("done", {"answer": "ok"})], prompt=300)]
    res = _run(replies, dispatch, max_steps=10)
    rw = next(s for s in res["steps"] if s["name"] == "rewind")
    assert rw.get("rejected") and rw["observed"].startswith("rewind refused")
    assert not res["rewinds"]
    tool_msgs = [m["content"] for m in res["messages"] if m.get("role") == "tool"]
    assert any(c.startswith("rewind refused") for c in tool_msgs)


def test_apply_runtime_validation():
    port = core.RuntimePort(owner="branch-0")
    assert core.apply_runtime("fork", {"tasks": ["x"]}, port)[0] == "fork needs at least two tasks"
    obs, _ = core.apply_runtime("fork", {"tasks": '["a", "b\\q"]'}, port)
    assert obs == core.FORK_STARTED + "branch-0.0, branch-0.1" and port.last_fork["branches"][1]["task"] == "b\\q"
    assert core.apply_runtime("commit", {"branch_id": "b"}, port)[0] == "commit needs branch_id and summary"
    assert core.apply_runtime("abort", {"branch_id": "b"}, port, needs=lambda n, a: "gated")[0] == "gated"
    assert core.apply_runtime("commit", {"branch_id": "b", "summary": "s"}, port)[0] == "commit recorded: b"
    assert core.cursor_delta([{"role": "user"}, {"cursor": "c1"}, {"role": "tool"}]) == ("c1", [{"role": "tool"}])
    assert core.cursor_delta([{"role": "user"}]) == (None, [{"role": "user"}])
