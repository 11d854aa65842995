"""Fork trees for branch-aware SFT, cut from logged episodes.

An episode log (`tree.json`, with `result.json` beside it) holds the main thread and,
per fork, the branch records.  Each fork that keeps at least `min_branches` branches
with a reply of their own, and after which the main thread replies again, becomes one
training tree:

* ``root``: the main thread before the fork, the context every branch started from.
  Only the episode's first tree trains its root (``train_root``); a later root repeats
  turns that an earlier tree's join child already trained.
* ``children``: the ``join`` child (the main thread from this fork up to the next kept
  fork, or to the end) and one ``branch`` child per kept branch (its task message and
  its own replies).

So every assistant turn of an episode is trained exactly once; a skipped fork's turns
are context of the next tree.

Reference parity (behaviour): `octopus/tools/tree_sft/trees.py:1-62`.
"""
from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path
from typing import Iterator


def _replies(msgs) -> bool:
    return any(m.get("role") == "assistant" for m in msgs)


def branch_turns(record: dict) -> list[dict]:
    """The messages a branch added itself: its history starts with the inherited prefix
    (``prefix_len`` messages, the last of which is its task message), so its own part
    starts at the task message."""
    msgs = record.get("messages") or []
    first_own = max(0, int(record.get("prefix_len", 1)) - 1)
    return msgs[first_own:]


@dataclass
class _KeptFork:
    at: int               # main-thread length when the fork was issued
    branches: list[dict]  # branch records that replied at least once


def _kept_forks(log: dict, min_branches: int) -> list[_KeptFork]:
    kept = []
    for rec in log.get("forks") or []:
        if "prefix_len" not in rec:
            continue
        live = [b for b in rec.get("branches") or [] if _replies(branch_turns(b))]
        if len(live) >= min_branches:
            kept.append(_KeptFork(int(rec["prefix_len"]), live))
    return kept


def fork_trees(log: dict, min_branches: int = 2) -> list[dict]:
    """Training trees of one episode log (see the module docstring)."""
    main = log.get("main") or []
    forks = _kept_forks(log, min_branches)
    stops = [f.at for f in forks[1:]] + [len(main)]
    trees: list[dict] = []
    for number, (fork, stop) in enumerate(zip(forks, stops)):
        join = main[fork.at:stop]
        if not _replies(join):
            continue
        children = [{"kind": "join", "messages": join}]
        children.extend({"kind": "branch", "branch_id": b["branch_id"], "messages": branch_turns(b)}
                        for b in fork.branches)
        trees.append({"fork_no": number, "tools": log.get("tools"), "root": main[:fork.at],
                      "train_root": len(trees) == 0, "children": children})
    return trees


def _episodes(log_dirs) -> Iterator[tuple[Path, dict, dict]]:
    """(episode folder, tree log, result) for every tree.json with a result.json beside it."""
    for base in log_dirs:
        for tree_file in sorted(Path(base).rglob("tree.json")):
            result_file = tree_file.with_name("result.json")
            if result_file.is_file():
                yield tree_file.parent, json.loads(tree_file.read_text()), json.loads(result_file.read_text())


def collect(log_dirs, min_reward: float | None = 1.0, min_branches: int = 2) -> list[dict]:
    """Trees of every logged episode below `log_dirs` whose reward is at least
    `min_reward` (None: all episodes, rewarded or not), tagged with task, trial folder
    and reward."""
    out = []
    for folder, log, result in _episodes(log_dirs):
        reward = result.get("reward")
        if min_reward is not None and (reward is None or reward < min_reward):
            continue
        task = result.get("task") or result.get("instance_id") or folder.name
        for tree in fork_trees(log, min_branches):
            out.append({**tree, "task": task, "trial": str(folder), "reward": reward})
    return out
