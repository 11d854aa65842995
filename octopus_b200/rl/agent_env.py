"""Agent-runtime RL environment: episodes of the cursor runtime (search / plan tasks,
forks, read_thread mounts) on the colocated engine, graded, credited and turned into
prefix-tree micro-batches by the workflow glue.

One rollout takes the next `batch_size` tasks, runs `n_samples` episodes per task
concurrently through the in-process chat service (requests from all episodes are
batched by the engine), grades each episode's final answer (y in {0, 1}), applies the
group credit (leave-one-out, branch gates), exports the per-leaf rows, drops groups
without reward variance and releases the episodes' cursors.

Reference parity (behaviour): the AReaL rollout workflow of `octopus/rl/workflow.py`
(EpisodeAgent.run -> plan_group_rewards -> _apply_plan) driven by
`octopus/rl/train.py:55-137`.
"""
from __future__ import annotations

import asyncio
import itertools
from dataclasses import dataclass, field

from ..runtime.core import branch_key, tree_branches
from ..runtime.tree import CursorRuntime
from .group import read_outcomes
from .workflow import TrainRow, plan_group_rewards, rows_to_microbatches


@dataclass
class AgentRollout:
    units: list = field(default_factory=list)       # per kept group: list[TrainRow]
    records: dict = field(default_factory=dict)
    generated_tokens: int = 0
    rewards: list = field(default_factory=list)
    episodes: list = field(default_factory=list)

    def microbatches(self, token_cap: int, build):
        return rows_to_microbatches(self.units, self.records, token_cap, build)


class AgentEnv:
    def __init__(self, chat, tasks: list[dict], make_workspace, grade, *, n_samples: int = 4, batch_size: int = 8,
                 branch_credit: str = "outcome", gate=None, filter_zero_variance: bool = True,
                 max_main_calls: int | None = None, branch_turns: int | None = None, grade_workspace: bool = False):
        """chat: async completion function (serving.local.ChatService); tasks: dicts with at
        least "question"; make_workspace(task) -> WorkspaceProvider; grade(task, answer) -> y,
        or with grade_workspace grade(task, answer, workspace, branch records) -> y (the
        episode's final tree decides, e.g. SWE tests; the grader may add fields to the branch
        records, which credit reads); a workspace with discard() is discarded after grading."""
        self.chat = chat
        self.tasks = tasks
        self._it = itertools.cycle(range(len(tasks)))
        self.make_workspace, self.grade = make_workspace, grade
        self.n, self.batch = n_samples, batch_size
        self.branch_credit, self.gate, self.filter = branch_credit, gate, filter_zero_variance
        self.max_main_calls, self.branch_turns = max_main_calls, branch_turns
        self.grade_workspace = grade_workspace
        self.step = 0

    async def _episodes(self, picked):
        async def one(ti, s):
            task = self.tasks[ti]
            ws = self.make_workspace(task)
            rt = CursorRuntime(ws, self.chat, session_id=f"r{self.step}-t{ti}-s{s}",
                               max_main_calls=self.max_main_calls, branch_turns=self.branch_turns)
            res = await rt.run(task["question"])
            if self.grade_workspace:
                branches = [br for _, _, br in tree_branches(res["tree"].get("forks") or [])]
                res["y"] = float(self.grade(task, res["tree"].get("answer"), ws, branches))
            if hasattr(ws, "discard"):
                ws.discard()
            return ti, res

        return await asyncio.gather(*[one(ti, s) for ti in picked for s in range(self.n)])

    def rollout(self, engine) -> AgentRollout:
        self.step += 1
        picked = [next(self._it) for _ in range(self.batch)]
        engine.record_interactions = True
        engine.records.clear()
        results = asyncio.run(self._episodes(picked))
        out = AgentRollout(records=dict(engine.records))
        groups: dict[int, list] = {}
        for ti, res in results:
            tree = res["tree"]
            branches = [{**br, "key": branch_key(name)} for name, _, br in tree_branches(tree.get("forks") or [])]
            y = res["y"] if "y" in res else float(self.grade(self.tasks[ti], tree.get("answer")))
            ep = {"y": y, "requests": res["requests"],
                  "branches": branches, "task": ti}
            ctl = tree.get("control")
            if ctl and "answer" in ctl and not self.grade_workspace:  # the main-first control's grade
                ep["control_y"] = float(self.grade(self.tasks[ti], ctl["answer"]))
            if tree.get("read_controls"):  # OCTOPUS_READ_CONTROL counterfactuals (credit on the read reply)
                ep["read_controls"] = [{k: v for k, v in c.items() if k != "result"} for c in tree["read_controls"]]
            groups.setdefault(ti, []).append(ep)
            out.episodes.append(ep)
            out.rewards.append(ep["y"])
            out.generated_tokens += sum(int(r["completion_tokens"]) for r in res["requests"])
        for eps in groups.values():
            rows: list[TrainRow] = plan_group_rewards(eps, out.records, self.branch_credit, self.gate, self.filter,
                                                      read_rewards=read_outcomes)
            if rows:
                out.units.append(rows)
        for rid in list(engine.records):
            if engine.cursors.get(rid) is not None:
                engine.release_cursor(rid)
        engine.records.clear()
        return out
