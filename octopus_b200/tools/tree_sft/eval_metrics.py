"""Branch-behaviour metrics of SWE runs, read from episode logs (a tree.json and a
result.json per episode, as `eval.swe_eval --log-dir` writes them).

    python -m octopus_b200.tools.tree_sft.eval_metrics --tasks TASK_TREES_DIR --run NAME=LOG_DIR [--run ...]

Per run (each a ratio; None when its denominator is empty):
  success         episodes with reward 1
  fork_rate       episodes that forked into >= 2 branches
  branch_close    branches that ended with commit or abort
  branch_overlap  mean Jaccard overlap of sibling branches' action sets (lower: a cleaner split)
  bug_coverage    forks where some branch viewed or edited a file of the reference fix
  join_redo       main-thread file views after a fork that re-open a file a branch viewed
  merge_ok        committed branch patches that merged at the join
File-level proxies (the reference fix's files come from TASK_TREES_DIR/<task>/solution/fix.patch):
  branch_hit      branches that viewed or edited a fix file
  branch_fix      editing branches whose edits touch a fix file
  select_ok       forks where a branch hit a fix file and the code changed after the join
                  (main-thread edits plus merged branch patches): those whose changes touch a
                  fix file
  select_branch   merged branch patches that came from a branch that hit a fix file

Reference parity (behaviour): `octopus/tools/tree_sft/eval_metrics.py:1-164` (the metric
set; the runtime here merges committed branch patches at the join itself, so merge_ok and
select_branch read the join's merge records instead of main-thread `git apply` calls).
"""
from __future__ import annotations

import argparse
import json
import re
from dataclasses import dataclass, field
from itertools import combinations
from pathlib import Path

from .trees import branch_turns

_FILE_TOOLS = ("view", "edit", "write")
_EDIT_TOOLS = ("edit", "write")


def _call_args(call: dict) -> dict:
    raw = (call.get("function") or {}).get("arguments")
    if isinstance(raw, dict):
        return raw
    try:
        parsed = json.loads(raw or "{}")
    except (TypeError, json.JSONDecodeError):
        return {}
    return parsed if isinstance(parsed, dict) else {}


def _norm_path(p) -> str:
    s = str(p or "").strip()
    if s.startswith("./"):
        s = s[2:]
    return s.lstrip("/") or "."


def action(call: dict) -> str:
    """A call as a comparable action: file tools by path, shell by command, reproduce by
    a hash of its code, other tools by name."""
    name, a = call["function"]["name"], _call_args(call)
    if name in _FILE_TOOLS:
        return f"{name}:{_norm_path(a.get('path'))}"
    if name == "shell":
        cmd = " ".join(str(a.get("cmd", a.get("command", ""))).split())
        return f"shell:{cmd[:200]}"
    if name == "reproduce":
        return f"reproduce:{hash(str(a.get('code', ''))) & 0xffffffff}"
    return name


def fix_files(tasks_dir, task: str) -> set[str]:
    """Files the task's reference fix changes (its '+++ b/<path>' headers)."""
    patch = Path(tasks_dir) / task / "solution" / "fix.patch"
    if not patch.is_file():
        return set()
    text = patch.read_text(errors="replace")
    return set(re.findall(r"^\+\+\+ b/(\S+)", text, re.M))


@dataclass
class _Calls:
    """The tool calls of a message list, with the file sets the metrics need."""

    calls: list[dict]

    @classmethod
    def of(cls, msgs) -> "_Calls":
        return cls([c for m in msgs if m.get("role") == "assistant" for c in m.get("tool_calls") or []])

    def files(self, tools) -> set[str]:
        return {_norm_path(_call_args(c).get("path")) for c in self.calls if c["function"]["name"] in tools}

    def actions(self) -> set[str]:
        return {action(c) for c in self.calls}


@dataclass
class _Ratios:
    """Named numerator / denominator pairs."""

    num: dict = field(default_factory=dict)
    den: dict = field(default_factory=dict)

    def add(self, name: str, hit, weight: float = 1.0):
        self.num[name] = self.num.get(name, 0.0) + float(hit)
        self.den[name] = self.den.get(name, 0.0) + weight

    def count(self, name: str) -> int:
        return int(self.den.get(name, 0))

    def value(self, name: str):
        d = self.den.get(name, 0.0)
        return round(self.num.get(name, 0.0) / d, 3) if d else None


def _score_fork(r: _Ratios, fork: dict, after_main: list[dict], later_main: list[dict], bug: set[str]):
    action_sets, touched, merged_edits = [], set(), set()
    for b in fork["branches"]:
        own = _Calls.of(branch_turns(b))
        seen, edited = own.files(_FILE_TOOLS), own.files(_EDIT_TOOLS)
        action_sets.append(own.actions())
        touched |= seen
        r.add("branch_close", b.get("ended_with") in ("commit", "abort"))
        if bug:
            r.add("branch_hit", bool(bug & seen))
            if edited:
                r.add("branch_fix", bool(bug & edited))
        if b.get("ended_with") == "commit" and (b.get("result") or {}).get("patch"):
            merged = b.get("merge") == "merged"
            r.add("merge_ok", merged)
            if merged:
                merged_edits |= edited
                r.add("select_branch", bool(bug & seen))
    for x, y in combinations(action_sets, 2):
        if x | y:
            r.add("branch_overlap", len(x & y) / len(x | y))
    changed = _Calls.of(after_main).files(_EDIT_TOOLS) | merged_edits
    if bug and bug & touched and changed:
        r.add("select_ok", bool(bug & changed))
    if bug:
        r.add("bug_coverage", bool(bug & touched))
    for c in _Calls.of(later_main).calls:
        if c["function"]["name"] == "view":
            r.add("join_redo", _norm_path(_call_args(c).get("path")) in touched)


def run_metrics(log_dir, tasks_dir) -> dict:
    r = _Ratios()
    forks_seen = 0
    for result_file in sorted(Path(log_dir).rglob("result.json")):
        result = json.loads(result_file.read_text())
        tree_file = result_file.with_name("tree.json")
        log = json.loads(tree_file.read_text()) if tree_file.is_file() else None
        r.add("success", result.get("reward") == 1.0)
        forks = [f for f in (log or {}).get("forks") or [] if len(f.get("branches") or []) >= 2]
        r.add("fork_rate", bool(forks))  # an episode without a log counts as not forked
        if log is None:
            continue
        main = log.get("main") or []
        bug = fix_files(tasks_dir, result.get("task") or result.get("instance_id") or "")
        for k, fork in enumerate(forks):
            forks_seen += 1
            start = fork.get("prefix_len", len(main))
            stop = forks[k + 1].get("prefix_len", len(main)) if k + 1 < len(forks) else len(main)
            _score_fork(r, fork, main[start:stop], main[start:], bug)
    out = {"episodes": r.count("success"), "forks": forks_seen}
    for name in ("success", "fork_rate", "branch_close", "branch_overlap", "bug_coverage", "join_redo", "merge_ok",
                 "branch_hit", "branch_fix", "select_ok", "select_branch"):
        out[name] = r.value(name)
    out.update(merges=r.count("merge_ok"), editing_branches=r.count("branch_fix"), selections=r.count("select_ok"),
               branch_merged=r.count("select_branch"))
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m octopus_b200.tools.tree_sft.eval_metrics")
    ap.add_argument("--tasks", required=True, help="task trees (envs.swe.taskset.write_task_tree)")
    ap.add_argument("--run", action="append", required=True, help="NAME=LOG_DIR")
    args = ap.parse_args(argv)
    for spec in args.run:
        name, path = spec.split("=", 1)
        print(json.dumps({"model": name, **run_metrics(path, args.tasks)}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
