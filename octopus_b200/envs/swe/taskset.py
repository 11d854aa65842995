"""SWE task set: task specs, selection, workspace preparation and the verifiers.

A task row (JSONL) names a git repository and the ref of its buggy state, the issue
statement, the visible test command (may be empty), the hidden test command and the hidden
test files the branch removed (restored only for grading), and optionally the reference fix.

  select_task_specs   rows whose repository exists locally, minus holdout / excluded ids
  branch_setup_script the instance's buggy ref checked out as the only commit: the history
                      holds the answer (the fix, the hidden tests), so it goes
  INFRA_RESTORE       test-infrastructure edits of the agent (conftest.py, pytest / tox /
                      setup / pyproject config) are undone before grading: no fix needs them,
                      and such an edit can make the hidden tests pass without a fix
  verify              the hidden tests on the final tree (infrastructure restored, hidden
                      files put back; the tree is left as the agent left it): 1.0 / 0.0
  plan_verify         verify, plus each committed branch's patch alone on its fork-point
                      tree: the branch grades of gate credit
  write_task_tree     a task directory (task.json, instruction.md, tests/, solution/)
  build_bundles       k tasks of one repository as one plan episode (statements listed,
                      every task's hidden tests graded; reward = fraction solved)

Reference parity (behaviour): `octopus/envs/swe/taskset.py` (branch setup that replaces the
history, INFRA_RESTORE / hidden restore before grading, holdout and exclusion selection,
task tree rendering, plan and bundle verifiers), `octopus/envs/swe/data/build_bundles.py`.
"""
from __future__ import annotations

import json
import os
import random
import shlex
import shutil
import tempfile
from dataclasses import asdict, dataclass, field
from pathlib import Path

HOLDOUT_IDS = frozenset()  # ids never trained on (a site list; extend per deployment)

INFRA_RESTORE = r"""git diff --name-only HEAD | grep -E '(^|/)(conftest\.py|pytest\.ini|tox\.ini|setup\.cfg|pyproject\.toml)$' | while read -r f; do git checkout -q HEAD -- "$f" 2>/dev/null || { git rm -q -f --cached "$f" 2>/dev/null; rm -f "$f"; }; done
git ls-files --others --exclude-standard | grep -E '(^|/)conftest\.py$' | xargs -r rm -f
"""


@dataclass
class TaskSpec:
    instance_id: str
    repo: str                       # local git repository
    ref: str = "HEAD"               # the buggy state
    statement: str = ""
    test_cmd: str = ""              # visible tests (the agent's `test` tool)
    hidden_test_cmd: str = ""       # grading command
    hidden_files: dict = field(default_factory=dict)  # path -> content, written before grading
    fix_patch: str = ""             # reference fix (bundle check validity; never shown)
    tasks: list = field(default_factory=list)  # bundle: member specs (dicts)

    @staticmethod
    def from_row(row: dict) -> "TaskSpec":
        keys = TaskSpec.__dataclass_fields__
        return TaskSpec(**{k: v for k, v in row.items() if k in keys})


def load_rows(path) -> list[dict]:
    """Rows of a JSONL file, or of every *.jsonl file in a directory."""
    p = Path(path)
    files = sorted(p.glob("*.jsonl")) if p.is_dir() else [p]
    rows = []
    for f in files:
        rows += [json.loads(x) for x in f.read_text().splitlines() if x.strip()]
    return rows


def instance_org(instance_id: str) -> str:
    return instance_id.split("__", 1)[0]


def is_excluded(instance_id: str, excluded: set) -> bool:
    """An id is excluded by its own entry or its organisation's (`org__*`)."""
    return instance_id in excluded or f"{instance_org(instance_id)}__*" in excluded


def select_task_specs(rows, excluded=frozenset(), holdout=HOLDOUT_IDS, require_repo: bool = True) -> list[TaskSpec]:
    out = []
    for r in rows:
        s = TaskSpec.from_row(r)
        if s.instance_id in holdout or is_excluded(s.instance_id, set(excluded)):
            continue
        if require_repo and not os.path.isdir(os.path.join(s.repo, ".git")):
            continue
        out.append(s)
    return out


def branch_setup_script(ref: str) -> str:
    """Check out `ref` and make it the repository's only commit (runs once, idempotent)."""
    q = shlex.quote(ref)
    return (f"if [ ! -f .git/octopus_ready ]; then git checkout -q --force {q} && rm -rf .git && git init -q"
            " && git add -A && git -c user.name=octopus -c user.email=octopus@localhost commit -qm 'Initial commit'"
            " && touch .git/octopus_ready; fi && test -f .git/octopus_ready")


def prepare_workspace(spec: TaskSpec, executor=None, timeout: float = 120.0):
    """A GitWorkspace on a fresh copy of the task's repository at its buggy ref."""
    from .containers import LocalExec, run_command
    from .workspace import GitWorkspace

    d = tempfile.mkdtemp(prefix=f"octo-task-{spec.instance_id[:40]}-")
    dst = os.path.join(d, "repo")
    shutil.copytree(spec.repo, dst, symlinks=True)
    r = run_command(["bash", "-c", branch_setup_script(spec.ref)], cwd=dst, timeout=timeout)
    if r.code != 0:
        shutil.rmtree(d, ignore_errors=True)
        raise RuntimeError(f"branch setup of {spec.instance_id} failed: {r.output[-500:]}")
    ws = GitWorkspace(dst, spec.test_cmd or "true", executor=executor or LocalExec(sandbox=True), timeout=timeout)
    ws.task_dir = d
    ws.defer_close = True  # the episode's end keeps the trees for plan_verify; discard() removes them
    return ws


def _grade_tree(exec_, d: str, spec: TaskSpec, timeout: float) -> bool:
    """Hidden tests of `spec` on directory d after restoring test infrastructure."""
    r = exec_.run(INFRA_RESTORE, d, timeout)
    if r.code != 0:
        return False
    for rel, content in (spec.hidden_files or {}).items():
        p = os.path.join(d, rel)
        os.makedirs(os.path.dirname(p) or d, exist_ok=True)
        with open(p, "w") as f:
            f.write(content)
    cmd = spec.hidden_test_cmd or spec.test_cmd
    return bool(cmd) and exec_.run(cmd, d, timeout).code == 0


def _graded_copy(ws, d: str, spec: TaskSpec) -> bool:
    """Grade a copy of directory d (the agent's tree stays as it is)."""
    tmp = tempfile.mkdtemp(prefix="octo-grade-")
    try:
        dst = os.path.join(tmp, "t")
        shutil.copytree(d, dst, symlinks=True)
        return _grade_tree(ws.exec, dst, spec, ws.timeout)
    finally:
        shutil.rmtree(tmp, ignore_errors=True)


def verify(ws, spec: TaskSpec) -> float:
    """1.0 when the hidden tests pass on the main thread's final tree (bundles: the fraction of
    member tasks whose hidden tests pass)."""
    if spec.tasks:
        members = [TaskSpec.from_row(t) for t in spec.tasks]
        return sum(_graded_copy(ws, ws.root, m) for m in members) / len(members)
    return 1.0 if _graded_copy(ws, ws.root, spec) else 0.0


def plan_verify(ws, spec: TaskSpec, results: list[dict]) -> tuple[float, dict]:
    """(reward of the final tree, {branch: passed}) with each committed branch's patch applied
    alone on its fork-point tree."""
    from .workspace import _git

    grades = {}
    for res in results:
        b = res.get("branch")
        if not b or res.get("ended_with") != "commit" or not res.get("patch"):
            continue
        d = ws.dirs.get(b)
        tmp = tempfile.mkdtemp(prefix="octo-branch-")
        try:
            dst = os.path.join(tmp, "t")
            shutil.copytree(d, dst, symlinks=True)
            _git(["reset", "-q", "--hard", ws.base.get(b, "HEAD")], dst)  # the fork point
            _git(["clean", "-qfd"], dst)
            ok = _git(["apply", "--whitespace=nowarn", "-"], dst, check=False, inp=res["patch"].encode()).returncode == 0
            grades[b] = ok and _grade_tree(ws.exec, dst, spec, ws.timeout)
        finally:
            shutil.rmtree(tmp, ignore_errors=True)
    return verify(ws, spec), grades


def write_task_tree(root, spec: TaskSpec) -> Path:
    """A task directory: task.json (the spec without hidden parts), instruction.md,
    tests/test.sh + hidden files, solution/fix.patch."""
    d = Path(root) / spec.instance_id
    (d / "tests").mkdir(parents=True, exist_ok=True)
    pub = {k: v for k, v in asdict(spec).items() if k not in ("hidden_files", "fix_patch", "hidden_test_cmd")}
    (d / "task.json").write_text(json.dumps(pub, indent=1))
    (d / "instruction.md").write_text(spec.statement + "\n")
    (d / "tests" / "test.sh").write_text("#!/bin/bash\n" + INFRA_RESTORE + (spec.hidden_test_cmd or spec.test_cmd) +
                                         "\n")
    (d / "tests" / "test.sh").chmod(0o755)
    for rel, content in (spec.hidden_files or {}).items():
        p = d / "tests" / "hidden" / rel
        p.parent.mkdir(parents=True, exist_ok=True)
        p.write_text(content)
    if spec.fix_patch:
        (d / "solution").mkdir(exist_ok=True)
        (d / "solution" / "fix.patch").write_text(spec.fix_patch)
    return d


def build_bundles(specs: list[TaskSpec], k: int, seed: int = 0) -> list[TaskSpec]:
    """Bundles of k tasks sharing a repository and ref: one plan episode each, the members'
    statements listed, graded per member."""
    by: dict = {}
    for s in specs:
        by.setdefault((s.repo, s.ref), []).append(s)
    rng = random.Random(seed)
    out = []
    for (repo, ref), group in sorted(by.items()):
        group = sorted(group, key=lambda s: s.instance_id)
        rng.shuffle(group)
        for i in range(0, len(group) - k + 1, k):
            mem = group[i:i + k]
            statement = "\n\n".join(f"Task {j + 1} ({m.instance_id}):\n{m.statement}" for j, m in enumerate(mem))
            out.append(TaskSpec(instance_id="bundle__" + "+".join(m.instance_id for m in mem), repo=repo, ref=ref,
                                statement=statement, test_cmd=mem[0].test_cmd,
                                tasks=[asdict(m) for m in mem]))
    return out


__all__ = ["INFRA_RESTORE", "TaskSpec", "branch_setup_script", "build_bundles", "load_rows", "plan_verify",
           "prepare_workspace", "select_task_specs", "verify", "write_task_tree"]
