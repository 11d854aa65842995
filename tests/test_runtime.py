"""Agent DAG runtime with a scripted fake chat model (no network, no GPU)."""
import asyncio
import json

import pytest

from octopus_b200.runtime import core
from octopus_b200.runtime.tree import CursorRuntime, WorkspaceProvider, run_episode


def call(name, **args):
    return {"id": f"c-{name}", "type": "function", "function": {"name": name, "arguments": json.dumps(args)}}


class Scripted:
    """Replies per session id from scripts: each entry a (content, [tool calls])."""

    def __init__(self, scripts):
        self.scripts = {k: list(v) for k, v in scripts.items()}
        self.bodies = []
        self.n = 0

    def __call__(self, body):
        self.bodies.append(body)
        sid = body["session_id"]
        key = next(k for k in self.scripts if sid.endswith(k))
        content, calls = self.scripts[key].pop(0)
        self.n += 1
        prompt = sum(len(str(m.get("content", ""))) for m in body["messages"]) // 4 + 10
        return {"id": f"r{self.n}", "cursor": f"r{self.n}",
                "choices": [{"message": {"role": "assistant", "content": content, "tool_calls": calls or None}}],
                "usage": {"prompt_tokens": prompt, "completion_tokens": 20}}


def test_fork_join_done(tmp_path):
    chat = Scripted({
        "ep": [("plan", [call("fork", tasks=["look left", "look right"])]), ("final", [call("done", answer="42")])],
        "branch-0": [("ok", [call("commit", branch_id="branch-0", summary="left is clear")])],
        "branch-1": [("ok", [call("commit", branch_id="branch-1", summary="right has 42")])],
    })
    out = run_episode(WorkspaceProvider(), chat, "find the number", log_dir=str(tmp_path))
    tree = out["tree"]
    assert tree["main_end"] == "done" and tree["answer"] == "42"
    (fork,) = tree["forks"]
    assert [b["branch_id"] for b in fork["branches"]] == ["branch-0", "branch-1"]
    assert [b["summary"] for b in fork["branches"]] == ["left is clear", "right has 42"]
    threads = [r["thread"] for r in out["requests"]]
    assert threads.count("main") == 2 and "fork0/branch-0" in threads and "fork0/branch-1" in threads
    # the join note reached main's next request
    last_main = [b for b in chat.bodies if b["session_id"] == "ep"][-1]
    assert any("right has 42" in str(m.get("content")) for m in last_main["messages"])
    assert (tmp_path / "tree.json").exists() and (tmp_path / "requests.jsonl").exists()


def test_fork_alone_and_remind_once():
    chat = Scripted({
        "ep": [("thinking...", []),  # no tool call: reminded once
               ("both", [call("fork", tasks=["a", "b"]), call("done", answer="x")]),  # done refused
               ("end", [call("done", answer="y")])],
        "branch-0": [("", [call("abort", branch_id="branch-0")])],
        "branch-1": [("", [call("abort", branch_id="branch-1")])],
    })
    out = run_episode(WorkspaceProvider(), chat, "t")
    steps = out["main"]["steps"]
    assert out["main"]["reminded"] == 1
    refused = [s for s in steps if s.get("name") == "done" and s.get("rejected")]
    assert refused and core.FORK_ALONE.format("done") == refused[0]["observed"]
    assert out["tree"]["answer"] == "y"


def test_main_call_cap_and_commit_in_main():
    chat = Scripted({"ep": [("", [call("commit", branch_id="x", summary="s")])] * 5})
    out = run_episode(WorkspaceProvider(), chat, "t", max_main_calls=3)
    assert out["tree"]["main_end"] == "step cap"
    assert all("no effect in the main thread" in s["observed"] for s in out["main"]["steps"])


def test_fork_depth_limit(monkeypatch):
    monkeypatch.setenv("OCTOPUS_FORK_DEPTH", "1")
    chat = Scripted({
        "ep": [("", [call("fork", tasks=["a", "b"])]), ("", [call("done", answer="z")])],
        "branch-0": [("", [call("fork", tasks=["c", "d"])]), ("", [call("commit", branch_id="branch-0", summary="s")])],
        "branch-1": [("", [call("commit", branch_id="branch-1", summary="s")])],
    })
    out = run_episode(WorkspaceProvider(), chat, "t")
    b0 = out["tree"]["forks"][0]["branches"][0]
    assert b0["ended_with"] == "commit"
    assert any(r["thread"] == "fork0/branch-0" for r in out["requests"])


def test_cursor_mode_sends_only_delta(monkeypatch):
    monkeypatch.setenv("OCTOPUS_CURSOR", "1")
    chat = Scripted({"ep": [("", [call("fork", tasks=["a", "b"])]), ("", [call("done", answer="q")])],
                     "branch-0": [("", [call("commit", branch_id="branch-0", summary="s0")])],
                     "branch-1": [("", [call("commit", branch_id="branch-1", summary="s1")])]})
    run_episode(WorkspaceProvider(), chat, "t")
    mains = [b for b in chat.bodies if b["session_id"] == "ep"]
    assert "cursor" not in mains[0] and mains[1]["cursor"] == "r1"
    assert mains[1]["messages"][0]["role"] == "tool"  # only the delta after the cursor


def test_read_thread_mounts_other_thread(monkeypatch):
    monkeypatch.setenv("OCTOPUS_READ_TOOL", "1")
    chat = Scripted({
        "ep": [("", [call("fork", tasks=["a", "b"])]), ("", [call("done", answer="q")])],
        "branch-0": [("", [call("commit", branch_id="branch-0", summary="s0")])],
        "branch-1": [("", [call("read_thread", thread="branch-0")]),
                     ("", [call("commit", branch_id="branch-1", summary="s1")])],
    })
    run_episode(WorkspaceProvider(), chat, "t")
    b1 = [b for b in chat.bodies if b["session_id"].endswith("branch-1")]
    assert "mount" not in b1[0]
    assert b1[1]["mount"] and b1[1]["mount"][0][0].startswith("r")


def test_post_chat_retries(monkeypatch):
    import urllib.error
    import urllib.request

    calls = {"n": 0}

    class Resp:
        status = 200

        def __enter__(self):
            return self

        def __exit__(self, *a):
            return False

        def read(self):
            return json.dumps({"id": "ok", "usage": {}}).encode()

    def fake_urlopen(req, timeout=None):
        calls["n"] += 1
        if calls["n"] < 3:
            raise urllib.error.HTTPError(req.full_url, 503, "busy", {}, None)
        return Resp()

    monkeypatch.setattr(urllib.request, "urlopen", fake_urlopen)
    out = core.post_chat("http://127.0.0.1:1/v1/chat/completions", {"messages": []}, attempts=4,
                         sleep=lambda s: None)
    assert out["id"] == "ok" and calls["n"] == 3


def test_fork_task_list_lenient():
    assert core.fork_task_list('["a\\|b", "c"]') == ["a\\|b", "c"]
    assert core.fork_task_list('["x",\n "y"] trailing') == ["x", "y"]
    msg, _ = core.apply_runtime("fork", {"tasks": ["only one"]})
    assert msg.startswith("fork needs at least two")


def test_main_first_control_run(monkeypatch):
    """OCTOPUS_PLAN_CONTROL=1: after a forking episode, main's history up to its forking reply
    continues without forks (fork is refused) as thread "control", closed by done; its
    requests are logged under "control" and the tree records its answer."""
    monkeypatch.setenv("OCTOPUS_PLAN_CONTROL", "1")
    chat = Scripted({
        "control": [("try fork", [call("fork", tasks=["a", "b"])]), ("alone", [call("done", answer="c-ans")])],
        "branch-0": [("", [call("commit", branch_id="branch-0", summary="s0")])],
        "branch-1": [("", [call("commit", branch_id="branch-1", summary="s1")])],
        "ep": [("look", [call("note", text="x")]), ("split", [call("fork", tasks=["a", "b"])]),
               ("end", [call("done", answer="fork-ans")])],
    })
    out = run_episode(WorkspaceProvider(), chat, "t")
    tree = out["tree"]
    assert tree["answer"] == "fork-ans" and tree["control"]["answer"] == "c-ans"
    assert tree["control"]["kind"] == "main-first" and tree["control"]["calls_before"] == 1
    ctl = [b for b in chat.bodies if b["session_id"].endswith("control")]
    assert len(ctl) == 2 and all(m.get("content") != "split" for m in ctl[0]["messages"])
    assert [r["thread"] for r in out["requests"]].count("control") == 2


def test_group_stats_fork_minus_control():
    from octopus_b200.rl.group import plan_group_stats

    eps = [{"y": 1.0, "A_main": 0.5, "control_y": 0.0, "branches": []},
           {"y": 0.0, "A_main": -0.5, "control_y": 0.0, "branches": []}, {"y": 1.0, "A_main": 0.5, "branches": []}]
    st = plan_group_stats(eps)
    assert st["fork_minus_control"] == 0.5 and st["controls"] == 2


def test_fork_wall_from_logs(tmp_path, monkeypatch):
    """fork_wall: a logged forking episode with its control gives one pair; the fork's cost is
    its critical path, the control's its own requests plus main's before the fork."""
    import json

    from octopus_b200.tools.fork_wall import run

    monkeypatch.setenv("OCTOPUS_PLAN_CONTROL", "1")
    chat = Scripted({
        "control": [("alone", [call("done", answer="c")])],
        "branch-0": [("", [call("commit", branch_id="branch-0", summary="s0")])],
        "branch-1": [("", [call("commit", branch_id="branch-1", summary="s1")])],
        "ep": [("split", [call("fork", tasks=["a", "b"])]), ("end", [call("done", answer="f")])],
    })
    run_episode(WorkspaceProvider(), chat, "t", log_dir=str(tmp_path / "ep"))
    (tmp_path / "ep" / "result.json").write_text(json.dumps({"reward": 1.0, "control_reward": 0.0}))
    out = run([str(tmp_path)], "tokens")
    # fork: main 2 replies + the longest branch (1 reply) = 3 x 20 tokens; control: 0 before + 1 reply
    assert out["pairs"] == 1 and out["ratio_median"] == 3.0 and out["fork_cheaper"] == 0.0
    assert out["gain"] == 1.0 and out["gain_when_not"] == 1.0


def test_read_control_continues_without_the_mount(monkeypatch):
    """OCTOPUS_READ_CONTROL: a branch whose read mounted gets a continuation from the state
    before its mount request, without the mount; forks and reads are refused there; the
    record names the reader, its read reply and how the control ended."""
    monkeypatch.setenv("OCTOPUS_READ_TOOL", "1")
    monkeypatch.setenv("OCTOPUS_READ_CONTROL", "1")
    chat = Scripted({
        "readctl/fork0/branch-1": [("", [call("fork", tasks=["x", "y"]), call("read_thread", thread="branch-0")]),
                                   ("", [call("abort", branch_id="branch-1")])],
        "ep": [("", [call("fork", tasks=["a", "b"])]), ("", [call("done", answer="q")])],
        "branch-0": [("", [call("commit", branch_id="branch-0", summary="s0")])],
        "branch-1": [("", [call("read_thread", thread="branch-0")]),
                     ("", [call("commit", branch_id="branch-1", summary="s1")])],
    })
    out = run_episode(WorkspaceProvider(), chat, "t")
    (rc,) = out["tree"]["read_controls"]
    assert rc["of"] == "fork0-branch-1" and rc["read_calls"] == ["read_thread"] and rc["read_call"] == 0
    assert rc["end"] == "abort" and not rc["forked_after"] and rc["control_forked"]
    reader = [b for b in chat.bodies if b["session_id"] == "ep/fork0/branch-1"]
    ctl = [b for b in chat.bodies if "readctl" in b["session_id"]]
    assert reader[1].get("mount") and not any(b.get("mount") for b in ctl)
    # the control started from the reader's history as it stood at the mount request
    tools = [str(m["content"]) for m in ctl[0]["messages"] if m.get("role") == "tool"]
    assert tools[-4].startswith("read_thread: mounted")  # the reader's read, then the control's own turns:
    assert tools[-3].startswith("Forking is not available") and "not available in this thread" in tools[-2]
    assert rc["read_rid"] == next(r["id"] for r in out["requests"] if r["thread"] == "fork0/branch-1")
    assert all(r["thread"] == "readctl/fork0/branch-1" for r in out["requests"][-2:])
    # credit: the reader committed, its control aborted -> +1 on the read reply
    from octopus_b200.rl.group import read_outcomes, read_values
    branches = [{"key": "fork0-branch-1", "ended_with": "commit"}]
    assert read_values({"read_controls": [rc], "branches": branches}, read_outcomes) == {}  # it tried to fork
    clean = {**rc, "control_forked": False}
    assert read_values({"read_controls": [clean], "branches": branches}, read_outcomes)[rc["read_rid"]]["v"] == 1.0
