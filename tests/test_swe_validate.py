"""SWE task validation on CPU: a task whose hidden tests fail on the buggy tree and pass with
the reference fix is valid; one whose tests already pass (nop = 1), one whose fix does not
apply and one without a fix are not; the CLI writes the valid rows and a report."""
import json
import platform
import sys
from dataclasses import asdict

import pytest

from octopus_b200.envs.swe.containers import LocalExec
from octopus_b200.envs.swe.taskset import TaskSpec
from octopus_b200.envs.swe.validate import main, select_valid
from test_swe_taskset import HIDDEN, _repo

pytestmark = pytest.mark.skipif(platform.machine() != "x86_64", reason="x86_64 guard")
FIX = ("--- a/calc.py\n+++ b/calc.py\n@@ -1,5 +1,5 @@\n def add(a, b):\n-    return a - b\n+    return a + b\n \n \n"
       " def mul(a, b):\n")
BAD = FIX.replace("a - b", "a * b")
PASSING = "from calc import mul\nassert mul(2, 2) == 4\n"  # 2 + 2: passes on the buggy tree


def _specs(repo):
    mk = lambda iid, hidden, fix: TaskSpec(iid, repo, "HEAD", "fix add", "", f"{sys.executable} test_hidden.py",  # noqa: E731
                                           {"test_hidden.py": hidden}, fix_patch=fix)
    return [mk("org__ok-1", HIDDEN, FIX), mk("org__nop-1", PASSING, FIX), mk("org__badfix-1", HIDDEN, BAD),
            mk("org__nofix-1", HIDDEN, "")]


def test_select_valid(tmp_path):
    specs = _specs(_repo(tmp_path))
    valid, rows = select_valid(specs, LocalExec(sandbox=True), timeout=30, workers=2)
    by = {r["task"]: r for r in rows}
    assert [s.instance_id for s in valid] == ["org__ok-1"]
    assert by["org__ok-1"]["nop"] == 0.0 and by["org__ok-1"]["oracle"] == 1.0
    assert by["org__nop-1"]["nop"] == 1.0 and not by["org__nop-1"]["valid"]
    assert "does not apply" in by["org__badfix-1"]["error"]
    assert "no reference fix" in by["org__nofix-1"]["error"]


def test_cli(tmp_path):
    specs = _specs(_repo(tmp_path))
    src = tmp_path / "tasks.jsonl"
    src.write_text("".join(json.dumps(asdict(s)) + "\n" for s in specs))
    out, rep = tmp_path / "valid.jsonl", tmp_path / "report.json"
    assert main([str(src), "--out", str(out), "--report", str(rep), "--workers", "2", "--timeout", "30"]) == 0
    assert [json.loads(x)["instance_id"] for x in out.read_text().splitlines()] == ["org__ok-1"]
    assert set(json.loads(rep.read_text())) == {s.instance_id for s in specs}
