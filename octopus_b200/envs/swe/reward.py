"""SWE rewards: an episode succeeds when the task's tests pass on the final tree; branch
grades for gate credit (a branch that committed a merged, non-empty, passing change
keeps its advantage, others only the bad side: `rl.group.code_gate`).

Reference parity (behaviour): `octopus/envs/swe/reward.py` (tests as the verifier,
branch grades), `octopus/rl/group.py` (code gate).
"""
from __future__ import annotations

from ...rl.group import code_gate, group_step


def swe_outcome(workspace) -> float:
    r = workspace.exec.run(workspace.test_cmd, workspace.root, workspace.timeout)
    return 1.0 if r.code == 0 else 0.0


def grade_branch(result: dict) -> dict:
    return {"ended_with": result.get("ended_with"), "merge": result.get("merge", ""),
            "diffstat": result.get("diffstat", ""), "passed": bool(result.get("passed"))}


def swe_group_step(episodes: list[dict], branch_credit: str = "gate") -> list[dict]:
    return group_step(episodes, branch_credit, gate=code_gate if branch_credit == "gate" else None)
