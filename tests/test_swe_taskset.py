"""SWE task set and plan episodes on CPU: a scripted agent (reproduce, fork a branch that
fixes the bug and commits, done) on a prepared task copy; the hidden tests grade the final
tree and the branch's patch alone on its fork point; test-infrastructure edits are undone
before grading; selection, task trees and bundles."""
import json
import platform
import subprocess
import sys

import pytest

from octopus_b200.envs.swe.containers import LocalExec
from octopus_b200.envs.swe.rl import grade_episode
from octopus_b200.envs.swe.taskset import (TaskSpec, build_bundles, prepare_workspace, select_task_specs, verify,
                                           write_task_tree)
from octopus_b200.runtime.tree import run_episode
from test_runtime import Scripted, call

pytestmark = pytest.mark.skipif(platform.machine() != "x86_64", reason="x86_64 guard")
HIDDEN = "from calc import add\nassert add(2, 3) == 5\n"
HIDDEN_MUL = "from calc import mul\nassert mul(2, 3) == 6\n"


def _repo(tmp_path):
    d = tmp_path / "repo"
    d.mkdir()
    (d / "calc.py").write_text("def add(a, b):\n    return a - b\n\n\ndef mul(a, b):\n    return a + b\n")
    for c in (["init", "-q"], ["add", "-A"], ["-c", "user.name=t", "-c", "user.email=t@t", "commit", "-qm", "bug"]):
        subprocess.run(["git", *c], cwd=d, check=True, capture_output=True)
    return str(d)


def _spec(repo, iid="org__calc-1", hidden=HIDDEN):
    return TaskSpec(iid, repo, "HEAD", "add() subtracts; make it add.", "",
                    f"{sys.executable} test_hidden.py", {"test_hidden.py": hidden})


def test_plan_episode_graded_by_hidden_tests(tmp_path):
    spec = _spec(_repo(tmp_path))
    ws = prepare_workspace(spec, LocalExec(sandbox=True), timeout=30)
    assert "test_hidden.py" not in subprocess.run(["git", "ls-files"], cwd=ws.root, capture_output=True,
                                                  text=True).stdout
    chat = Scripted({
        "ep": [("repro", [call("reproduce", hypothesis="add subtracts", code="from calc import add; print(add(2, 3))")]),
               ("fork", [call("fork", tasks=["fix add", "look at mul"])]), ("end", [call("done", answer="fixed")])],
        "branch-0": [("rerun", [call("rerun_reproduction")]),
                     ("edit", [call("edit", path="calc.py", old="a - b", new="a + b")]),
                     ("ok", [call("commit", branch_id="branch-0", summary="add fixed")])],
        "branch-1": [("no", [call("abort", branch_id="branch-1", reason="out of scope")])],
    })
    out = run_episode(ws, chat, spec.statement)
    steps = out["main"]["steps"]
    assert steps[0]["name"] == "reproduce" and "-1" in steps[0]["observed"]
    (fork,) = out["tree"]["forks"]
    branches = fork["branches"]
    y = grade_episode({"spec": spec}, out["tree"]["answer"], ws, branches)
    assert y == 1.0 and branches[0]["passed"] and "calc.py" in branches[0]["diffstat"]
    assert not branches[1]["passed"]
    # grading leaves the agent's tree as it was (no hidden file written into it)
    assert not __import__("os").path.exists(f"{ws.root}/test_hidden.py")
    ws.discard()


def test_infra_edits_undone_and_bundles(tmp_path):
    repo = _repo(tmp_path)
    spec = _spec(repo)
    ws = prepare_workspace(spec, LocalExec(sandbox=True), timeout=30)
    # an agent "fix" that only adds a conftest.py is undone before grading
    with open(f"{ws.root}/conftest.py", "w") as f:
        f.write("raise SystemExit(0)\n")
    assert verify(ws, spec) == 0.0
    with open(f"{ws.root}/calc.py", "w") as f:
        f.write("def add(a, b):\n    return a + b\n\n\ndef mul(a, b):\n    return a + b\n")
    assert verify(ws, spec) == 1.0
    ws.discard()
    s2 = _spec(repo, "org__calc-2", HIDDEN_MUL)
    (b,) = build_bundles([spec, s2], 2)
    assert len(b.tasks) == 2 and "Task 2" in b.statement
    ws = prepare_workspace(b, LocalExec(sandbox=True), timeout=30)
    with open(f"{ws.root}/calc.py", "w") as f:
        f.write("def add(a, b):\n    return a + b\n\n\ndef mul(a, b):\n    return a + b\n")
    assert verify(ws, b) == 0.5
    ws.discard()
    sel = select_task_specs([json.loads(json.dumps(spec.__dict__)), {**s2.__dict__, "instance_id": "bad__x"},
                             {**s2.__dict__, "repo": str(tmp_path / "missing")}], excluded={"bad__*"})
    assert [s.instance_id for s in sel] == ["org__calc-1"]
    d = write_task_tree(tmp_path / "tasks", spec)
    assert (d / "instruction.md").read_text().startswith("add()") and (d / "tests/hidden/test_hidden.py").exists()
    assert "hidden_test_cmd" not in json.loads((d / "task.json").read_text())
