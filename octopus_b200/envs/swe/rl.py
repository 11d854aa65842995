"""SWE plan episodes for RL: a task's issue statement is the main thread's task; the agent
(main + free forks) works in a prepared copy of the task's repository; the episode is
scored on its final tree by the hidden tests (R = 2y - 1 in the group credit), and each
committed branch's patch alone on its fork-point tree gives the branch grade of gate credit.

Reference parity (behaviour): `octopus/envs/swe/rl.py:1-40` (one plan episode per task,
pure outcome on the final tree, branch grades from the plan verifier, infrastructure
failures raise instead of training), `octopus/envs/swe/reward.py`.
"""
from __future__ import annotations

from ...rl.agent_env import AgentEnv
from ...rl.group import code_gate
from .taskset import TaskSpec, plan_verify, prepare_workspace


def grade_episode(task: dict, answer, ws, branches: list[dict]) -> float:
    """y of the episode; the branch records get `passed` (their patch alone on the fork-point
    tree passes the hidden tests) and `diffstat` for gate credit."""
    results = [{**(br.get("result") or {}), "branch": br.get("thread"), "ended_with": br.get("ended_with")}
               for br in branches]
    y, grades = plan_verify(ws, task["spec"], results)
    for br in branches:
        br["passed"] = bool(grades.get(br.get("thread"), False))
        br["diffstat"] = (br.get("result") or {}).get("diffstat", "")
    return y


def swe_agent_env(chat, specs: list[TaskSpec], executor=None, *, n_samples: int = 4, batch_size: int = 8,
                  branch_credit: str = "gate", timeout: float = 120.0, **kw) -> AgentEnv:
    """An AgentEnv over SWE task specs (rl.agent_env: rollout -> prefix-tree micro-batches)."""
    tasks = [{"question": s.statement, "spec": s} for s in specs]
    return AgentEnv(chat, tasks, lambda t: prepare_workspace(t["spec"], executor, timeout), grade_episode,
                    n_samples=n_samples, batch_size=batch_size, branch_credit=branch_credit,
                    gate=code_gate if branch_credit == "gate" else None, grade_workspace=True, **kw)


__all__ = ["grade_episode", "swe_agent_env"]
