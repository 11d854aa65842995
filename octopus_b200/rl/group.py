"""Group credit of tree episodes: outcome reward, leave-one-out baseline, branch credit,
single ownership of every generated token, and critical-path costs.

* R = 2y - 1 per episode; A_main = leave-one-out over the group (no std): the mean of
  the differences to the other episodes, exactly 0 when all are equal.
* Every branch thread takes its episode's A_main ("outcome"), or an environment gate
  ("gate": an ok branch keeps A, another only its bad side min(A, 0)).
* Single ownership: every request's completion is trained by exactly one exported
  leaf; a thread's requests after its last leaf (its last request forked) are adopted
  by the first leaf of its first branch, at their own thread's advantage (a span).
* Critical path: the tree's longest chain of dependent work (completion tokens, model
  calls or wall seconds), overlapping forks counted once.

Reference parity: `octopus/rl/group.py:36-433` (leave_one_out, group_step,
tree_advantage, assign_threads, critical_path, plan_group_stats).
"""
from __future__ import annotations

import re
from collections import defaultdict

from ..runtime.core import branch_key


def leave_one_out(values: list[float]) -> list[float]:
    """A_i = x_i - mean_{j != i} x_j computed as mean_j (x_i - x_j) over j != i."""
    n = len(values)
    if n < 2:
        return [0.0] * n
    return [sum(x - v for v in values) / (n - 1) for x in values]


def group_step(episodes: list[dict], branch_credit: str = "outcome", gate=None, read_rewards=None) -> list[dict]:
    """Fill R, A_main on each episode and A_branch on each of its branches (in place)."""
    if branch_credit not in ("outcome", "gate"):
        raise ValueError(f"branch_credit {branch_credit!r}: outcome or gate")
    if branch_credit == "gate" and gate is None:
        raise ValueError("branch_credit=gate needs the environment's gate rule")
    for e in episodes:
        e["R"] = 2.0 * float(e["y"]) - 1.0
    for e, a in zip(episodes, leave_one_out([e["R"] for e in episodes])):
        e["A_main"] = a
        for b in e.get("branches") or []:
            b["A_branch"] = gate(a, b) if branch_credit == "gate" else a
    if read_rewards is not None:
        for e in episodes:
            e["read_adv"] = read_values(e, read_rewards)
    return episodes


def read_outcomes(episode: dict, control: dict, branch: dict) -> tuple[float, float]:
    """Default read-control rewards: 1 for a branch (the reader, or its control) that closed
    with commit, else 0.  Environments that grade branch results can pass their own."""
    return float(branch.get("ended_with") == "commit"), float(control.get("end") == "commit")


def read_values(episode: dict, read_rewards) -> dict:
    """Read-control counterfactual: {reader reply id: {calls, call, v = r_reader - r_control}}."""
    out = {}
    for c in episode.get("read_controls") or []:
        if c.get("forked_after") or c.get("control_forked"):
            continue
        b = next(x for x in episode["branches"] if x["key"] == c["of"])
        r_reader, c["r"] = read_rewards(episode, c, b)
        calls = c["read_calls"]
        reads = [k for k, name in enumerate(calls) if name == "read_thread"]
        out[c["read_rid"]] = {"calls": calls, "v": r_reader - c["r"], "call": reads[c.get("read_call", 0)]}
    return out


def search_gate(a: float, branch: dict) -> float:
    ok = branch.get("ended_with") == "done" and bool(str(branch.get("summary") or "").strip()) and \
        (branch.get("searched") or 0) > 0
    return a if ok else min(a, 0.0)


def code_gate(a: float, branch: dict) -> float:
    ok = (branch.get("ended_with") == "commit" and str(branch.get("merge") or "").startswith("merged")
          and bool(branch.get("diffstat")) and bool(branch.get("passed")))
    return max(a, 0.0) if ok else min(a, 0.0)


def _is_child_thread(parent: str, name: str) -> bool:
    prefix = "" if parent == "main" else parent + "/"
    return re.fullmatch(re.escape(prefix) + r"fork\d+/[^/]+", name) is not None


def assign_threads(leaf_ids: list[str], episode: dict) -> dict:
    """Ownership of every request's completion by exactly one leaf.

    episode["requests"]: [(response id, thread, prompt_tokens, completion_tokens)] in order.
    Returns {leaf id: {"adv", "own_start", "spans"}}; raises when a request has no owner.
    """
    reqs = episode["requests"]
    thread_of = {rid: th for rid, th, _, _ in reqs}
    missing = set(leaf_ids) - set(thread_of)
    if missing:
        raise RuntimeError(f"no request row for leaf {sorted(missing)[0]}")
    owner: dict[int, str] = {}
    last: dict[str, int] = {}
    leaves = set(leaf_ids)
    for i, (rid, th, _, _) in enumerate(reqs):
        if rid in leaves:
            for j in range(last.get(th, -1) + 1, i + 1):
                if reqs[j][1] == th:
                    owner[j] = rid
            last[th] = i

    def adopt(i: int) -> str:
        th = reqs[i][1]
        final = max(j for j, r in enumerate(reqs) if r[1] == th)
        child = next((j for j in range(final + 1, len(reqs)) if _is_child_thread(th, reqs[j][1])), None)
        if child is None:
            raise RuntimeError(f"request {reqs[i][0]} of {th} belongs to no leaf and no branch extends it")
        return owner[child] if child in owner else adopt(child)

    for i, (_, th, _, _) in enumerate(reqs):
        if i not in owner and not th.startswith("readctl/") and th != "control":
            owner[i] = adopt(i)
    branches = {b["key"]: b for b in episode.get("branches") or []}

    def adv(th: str) -> float:
        if th == "main":
            return episode["A_main"]
        b = branches.get(branch_key(th))
        if b is None:
            raise RuntimeError(f"branch thread {th} has no graded branch")
        return b["A_branch"]

    out = {}
    for lid in leaf_ids:
        th = thread_of[lid]
        if th.startswith("readctl/") or th == "control":
            out[lid] = {"reward": episode["R"], "adv": 0.0, "own_start": None, "spans": []}
            continue
        a = adv(th)
        own = [(reqs[j], adv(reqs[j][1])) for j in sorted(owner) if owner[j] == lid]
        row = {"reward": episode["R"], "adv": a, "own_start": own[0][0][2] if own else None, "spans": []}
        for (rid, t2, p, c), a2 in own:
            if t2 != th:
                row["spans"].append((p, p + c, a2 - a))
        out[lid] = row
    return out


def critical_path(requests: list[dict], unit: str = "tokens") -> float:
    """Longest dependent chain from main: a thread's own work in order plus, per fork, its
    longest branch (branches of one fork overlap).  requests: rows with "thread" and
    "completion_tokens" (unit tokens), "id" (unit calls) or "elapsed_s" (unit wall)."""
    own = defaultdict(float)
    for r in requests:
        th = r.get("thread") or "main"
        if th == "control" or th.startswith("readctl/"):
            continue
        if unit == "tokens":
            own[th] += float(r.get("completion_tokens") or 0)
        elif unit == "calls":
            own[th] += 1.0 if r.get("id") else 0.0
        else:
            own[th] += float(r.get("elapsed_s") or 0)

    def path(th: str) -> float:
        forks = defaultdict(float)
        for child in list(own):
            if child != th and _is_child_thread(th, child):
                fk = child.rsplit("/", 1)[0]
                forks[fk] = max(forks[fk], path(child))
        return own.get(th, 0.0) + sum(forks.values())

    return path("main")


def plan_group_stats(episodes: list[dict]) -> dict:
    def mean(xs):
        return round(sum(xs) / len(xs), 4) if xs else None

    rows = [b for e in episodes for b in e.get("branches") or []]
    ctl = [e for e in episodes if e.get("control_y") is not None]
    return {"abs_A_main": mean([abs(e["A_main"]) for e in episodes]),
            "abs_A_branch": mean([abs(b["A_branch"]) for b in rows]),
            "y": mean([float(e["y"]) for e in episodes]),
            "forked": mean([float(bool(e.get("forked"))) for e in episodes]),
            # fork vs its main-first control (OCTOPUS_PLAN_CONTROL): y - y_control
            "fork_minus_control": mean([float(e["y"]) - float(e["control_y"]) for e in ctl]),
            "controls": len(ctl)}


def has_variance(rewards: list[float]) -> bool:
    """Dynamic filter: a group whose rewards are all equal carries no advantage."""
    return len(set(float(r) for r in rewards)) > 1
