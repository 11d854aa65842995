"""Fork trees for branch-aware SFT from episode logs.

A tree is one fork of one episode:
  root      the main thread's messages up to the fork (the history every branch resumed
            from); its assistant turns are trained only in the episode's first tree
            (`train_root`): later trees' roots repeat turns an earlier join child trained
  children  "join": the main thread from the fork to the next kept fork (or the end): the
            join note and the turns after it; "branch": one per branch with turns, its
            task message and its own turns
Every assistant turn of an episode is trained once.  Forks with fewer than `min_branches`
branches with turns, or with no main-thread turn after them, are skipped (their turns stay
context of the next tree).

Reference parity (behaviour): `octopus/tools/tree_sft/trees.py:1-62`.
"""
from __future__ import annotations

import json
from pathlib import Path


def _own(br: dict) -> list[dict]:
    """A branch record's own messages (task message + its turns); its history holds the
    inherited prefix first."""
    msgs = br.get("messages") or []
    return msgs[max(0, int(br.get("prefix_len", 1)) - 1):]


def fork_trees(tree: dict, min_branches: int = 2) -> list[dict]:
    main, forks = tree.get("main") or [], tree.get("forks") or []
    kept = []
    for fork in forks:
        branches = [b for b in fork.get("branches") or [] if any(m.get("role") == "assistant" for m in _own(b))]
        if len(branches) >= min_branches and "prefix_len" in fork:
            kept.append((fork, branches))
    out = []
    for i, (fork, branches) in enumerate(kept):
        start = fork["prefix_len"]
        end = kept[i + 1][0]["prefix_len"] if i + 1 < len(kept) else len(main)
        join = main[start:end]
        if not any(m.get("role") == "assistant" for m in join):
            continue
        out.append({"fork_no": i, "tools": tree.get("tools"), "root": main[:start], "train_root": not out,
                    "children": [{"kind": "join", "messages": join}] +
                    [{"kind": "branch", "branch_id": b["branch_id"], "messages": _own(b)} for b in branches]})
    return out


def collect(log_dirs, min_reward: float | None = 1.0, min_branches: int = 2) -> list[dict]:
    """Trees of every episode below `log_dirs` (a tree.json beside a result.json with
    "reward") whose reward is at least min_reward (None: every episode)."""
    trees = []
    for d in log_dirs:
        for log in sorted(Path(d).rglob("tree.json")):
            res_f = log.parent / "result.json"
            if not res_f.is_file():
                continue
            res = json.loads(res_f.read_text())
            reward = res.get("reward")
            if min_reward is not None and (reward is None or reward < min_reward):
                continue
            for t in fork_trees(json.loads(log.read_text()), min_branches):
                t.update({"task": res.get("task") or res.get("instance_id") or log.parent.name,
                          "trial": str(log.parent), "reward": reward})
                trees.append(t)
    return trees
