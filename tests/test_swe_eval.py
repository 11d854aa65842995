"""SWE dev evaluation on CPU: two tasks through the eval's episode runner with a scripted
chat; one episode fixes the bug in a committed branch (a second branch aborts), the other ends without a fix.  The
summary's resolve rate, pass@1 and branch pass rate come from the hidden tests."""
import platform
import sys

import pytest

from octopus_b200.envs.swe.containers import LocalExec
from octopus_b200.envs.swe.taskset import TaskSpec
from octopus_b200.eval.swe_eval import evaluate
from test_runtime import Scripted, call
from test_swe_taskset import HIDDEN, _repo

pytestmark = pytest.mark.skipif(platform.machine() != "x86_64", reason="x86_64 guard")


class _Routed(Scripted):
    """Scripts keyed by "task:thread": a branch's session id ends with "/<branch id>"."""

    def __call__(self, body):
        sid = body["session_id"]
        task = "calc-1" if "calc-1" in sid else "calc-2"
        thread = sid.rsplit("/", 1)[-1] if "/" in sid else "main"
        body = {**body, "session_id": f"{task}:{thread}"}
        return super().__call__(body)


def test_swe_eval_resolve_rate(tmp_path):
    repo = _repo(tmp_path)
    specs = [TaskSpec(f"org__calc-{i}", repo, "HEAD", "add() subtracts; make it add.", "",
                      f"{sys.executable} test_hidden.py", {"test_hidden.py": HIDDEN}) for i in (1, 2)]
    chat = _Routed({
        "calc-1:main": [("fork", [call("fork", tasks=["fix add", "look at mul"])]),
                        ("end", [call("done", answer="fixed")])],
        "calc-1:branch-0": [("edit", [call("edit", path="calc.py", old="a - b", new="a + b")]),
                            ("ok", [call("commit", branch_id="branch-0", summary="add fixed")])],
        "calc-1:branch-1": [("no", [call("abort", branch_id="branch-1", reason="out of scope")])],
        "calc-2:main": [("end", [call("done", answer="nothing to do")])],
    })

    class Svc:
        pass

    svc = Svc()
    svc.chat = chat
    out = evaluate(svc, specs, samples=1, executor=LocalExec(sandbox=True), timeout=30)
    rows = {r["instance_id"]: r for r in out["rows"]}
    assert rows["org__calc-1"]["resolved"] and rows["org__calc-1"]["branches"] == 2
    assert rows["org__calc-1"]["branches_passed"] == 1
    assert not rows["org__calc-2"]["resolved"] and rows["org__calc-2"]["branches"] == 0
    s = out["summary"]
    assert s["tasks"] == 2 and s["episodes"] == 2 and s["resolved"] == 0.5 and s["pass@1"] == 0.5
    assert s["branch_pass_rate"] == 0.5 and s["mean_critical_path"] > 0
