"""Branch-behaviour metrics of SWE runs from episode logs (tree.json + result.json per
episode, as `eval.swe_eval --log-dir` writes them).

    python -m octopus_b200.tools.tree_sft.eval_metrics --tasks TASK_TREES_DIR --run NAME=LOG_DIR [--run ...]

Per run:
  success         share of episodes with reward 1
  fork_rate       share of episodes with a fork into >= 2 branches
  branch_close    share of branches that ended with commit or abort
  branch_overlap  mean Jaccard overlap of sibling branches' actions (lower: a cleaner split)
  bug_coverage    share of forks where some branch viewed or edited a file of the reference fix
  join_redo       share of the main thread's post-join file views that re-open a file a
                  branch viewed
  merge_ok        share of committed branch patches that merged at the join
File-level proxies (reference fix files from TASK_TREES_DIR/<task>/solution/fix.patch):
  branch_hit      share of branches that viewed or edited a fix file
  branch_fix      share of editing branches whose edits touch a fix file
  select_ok       forks where some branch hit a fix file and the code changed after the join
                  (main-thread edits plus merged branch patches): share whose changes touch a
                  fix file
  select_branch   merged branch patches: share from a branch that hit a fix file

Reference parity (behaviour): `octopus/tools/tree_sft/eval_metrics.py:1-164` (the metric
set; the runtime here merges committed branch patches at the join itself, so merge_ok and
select_branch read the join's merge records instead of main-thread `git apply` calls).
"""
from __future__ import annotations

import argparse
import json
import re
from collections import defaultdict
from itertools import combinations
from pathlib import Path


def _args(call: dict) -> dict:
    raw = (call.get("function") or {}).get("arguments")
    if isinstance(raw, dict):
        return raw
    try:
        v = json.loads(raw or "{}")
        return v if isinstance(v, dict) else {}
    except (TypeError, json.JSONDecodeError):
        return {}


def _path(p) -> str:
    p = re.sub(r"^\./", "", str(p or "").strip())
    return p.lstrip("/") or "."


def action(call: dict) -> str:
    name, a = call["function"]["name"], _args(call)
    if name in ("view", "edit", "write"):
        return f"{name}:{_path(a.get('path'))}"
    if name == "shell":
        return "shell:" + " ".join(str(a.get("cmd", a.get("command", ""))).split())[:200]
    if name == "reproduce":
        return f"reproduce:{hash(str(a.get('code', ''))) & 0xffffffff}"
    return name


def fix_files(tasks_dir, task: str) -> set[str]:
    patch = Path(tasks_dir) / task / "solution" / "fix.patch"
    if not patch.is_file():
        return set()
    return {m.group(1) for m in re.finditer(r"^\+\+\+ b/(\S+)", patch.read_text(errors="replace"), re.M)}


def _calls(msgs) -> list[dict]:
    return [c for m in msgs if m.get("role") == "assistant" for c in (m.get("tool_calls") or [])]


def _files(calls, names) -> set[str]:
    return {_path(_args(c).get("path")) for c in calls if c["function"]["name"] in names}


def run_metrics(log_dir, tasks_dir) -> dict:
    s = defaultdict(float)
    for res_f in sorted(Path(log_dir).rglob("result.json")):
        res = json.loads(res_f.read_text())
        s["episodes"] += 1
        s["success"] += res.get("reward") == 1.0
        tree_f = res_f.parent / "tree.json"
        if not tree_f.is_file():
            continue
        tree = json.loads(tree_f.read_text())
        main = tree.get("main") or []
        bug = fix_files(tasks_dir, res.get("task") or res.get("instance_id") or "")
        forks = [f for f in tree.get("forks") or [] if len(f.get("branches") or []) >= 2]
        s["forked"] += bool(forks)
        for fi, f in enumerate(forks):
            s["forks"] += 1
            acts, touched, merged_files, hit_merged = [], set(), set(), 0
            merges = 0
            for b in f["branches"]:
                s["branches"] += 1
                s["branch_closed"] += b.get("ended_with") in ("commit", "abort")
                calls = _calls((b.get("messages") or [])[max(0, int(b.get("prefix_len", 1)) - 1):])
                acts.append({action(c) for c in calls})
                seen, edited = _files(calls, ("view", "edit", "write")), _files(calls, ("edit", "write"))
                touched |= seen
                if bug:
                    s["branches_with_bug_files"] += 1
                    s["branch_hit"] += bool(bug & seen)
                    if edited:
                        s["editing_branches"] += 1
                        s["branch_fix"] += bool(bug & edited)
                if b.get("ended_with") == "commit" and (b.get("result") or {}).get("patch"):
                    s["merges"] += 1
                    ok = b.get("merge") == "merged"
                    s["merge_ok"] += ok
                    if ok:
                        merges += 1
                        merged_files |= edited
                        hit_merged += bool(bug & seen)
            s["branch_merged"] += merges
            s["select_branch"] += hit_merged
            start = f.get("prefix_len", len(main))
            end = forks[fi + 1].get("prefix_len", len(main)) if fi + 1 < len(forks) else len(main)
            after = _calls(main[start:end])
            changed = _files(after, ("edit", "write")) | merged_files
            if bug and bug & touched and changed:
                s["selections"] += 1
                s["select_ok"] += bool(bug & changed)
            for x, y in combinations(acts, 2):
                if x | y:
                    s["pairs"] += 1
                    s["overlap"] += len(x & y) / len(x | y)
            s["bug_covered"] += bool(bug & touched)
            s["forks_with_bug_files"] += bool(bug)
            for c in _calls(main[start:]):
                if c["function"]["name"] == "view":
                    s["join_views"] += 1
                    s["join_redo"] += _path(_args(c).get("path")) in touched

    def ratio(a, b):
        return round(s[a] / s[b], 3) if s[b] else None
    return {"episodes": int(s["episodes"]), "success": ratio("success", "episodes"),
            "fork_rate": ratio("forked", "episodes"), "forks": int(s["forks"]),
            "branch_close": ratio("branch_closed", "branches"), "branch_overlap": ratio("overlap", "pairs"),
            "bug_coverage": ratio("bug_covered", "forks_with_bug_files"), "join_redo": ratio("join_redo", "join_views"),
            "merge_ok": ratio("merge_ok", "merges"), "merges": int(s["merges"]),
            "branch_hit": ratio("branch_hit", "branches_with_bug_files"),
            "branch_fix": ratio("branch_fix", "editing_branches"), "editing_branches": int(s["editing_branches"]),
            "select_ok": ratio("select_ok", "selections"), "selections": int(s["selections"]),
            "select_branch": ratio("select_branch", "branch_merged"), "branch_merged": int(s["branch_merged"])}


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
