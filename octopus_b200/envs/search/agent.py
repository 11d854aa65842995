"""Search agent workspace: tools ``search``, ``open`` and ``done`` over a retrieval
backend, no file workspace; branches (depth 1 by default) close with ``done`` too and
hand their answer back as the summary.

Defaults per question: main's calls 100, a branch's turns 50, at most 10 branches,
only main forks, answer reserve 2048 (set as OCTOPUS_* switches by `search_defaults`).

Reference parity (behaviour): `octopus/envs/search/agent.py:143-291`,
`octopus/envs/search/defaults.py`.
"""
from __future__ import annotations

import json
import os

from ...runtime.core import DONE_TOOL, _tool
from ...runtime.tree import WorkspaceProvider

DEFAULTS = {"OCTOPUS_MAIN_MAX_CALLS": "100", "OCTOPUS_BRANCH_MAX_TURNS": "50", "OCTOPUS_SEARCH_BUDGET": "0",
            "OCTOPUS_MAX_BRANCHES": "10", "OCTOPUS_FORK_DEPTH": "1", "OCTOPUS_ANSWER_RESERVE": "2048"}

SEARCH_TOOL = _tool("search", "Search the corpus; returns the top documents with snippets.",
                    {"query": {"type": "string"}, "k": {"type": "integer"}}, ["query"])
OPEN_TOOL = _tool("open", "Open a document by id; returns one page of its text.",
                  {"docid": {"type": "string"}, "page": {"type": "integer"}}, ["docid"])


def search_defaults(env=None) -> dict:
    env = os.environ if env is None else env
    for k, v in DEFAULTS.items():
        env.setdefault(k, v)
    return {k: env[k] for k in DEFAULTS}


class SearchWorkspace(WorkspaceProvider):
    report = "the answer you found and the evidence"

    def __init__(self, retrieval, question: str, k: int = 10):
        self.retrieval = retrieval
        self.question = question
        self.k = k
        self.searched: dict[str, int] = {}
        self.opened: set[str] = set()   # docids opened in the episode (evidence recall)

    def system_prompt(self, task: str) -> str:
        return ("You answer a research question with a search tool over a document corpus. Use search and open, "
                "fork parallel branches for independent sub-questions, and call done with the final answer.")

    def tools(self):
        return [SEARCH_TOOL, OPEN_TOOL, DONE_TOOL]

    def budget(self):
        b = int(os.environ.get("OCTOPUS_SEARCH_BUDGET", "0") or 0)
        return b or None

    def closing(self, depth: int) -> set:
        return {"done"}

    def fork_min(self) -> int:
        return 1

    async def dispatch(self, name, args, thread):
        if name == "search":
            self.searched[thread] = self.searched.get(thread, 0) + 1
            res = self.retrieval.search(str(args.get("query", "")), int(args.get("k", self.k)))
            return json.dumps(res), False
        if name == "open":
            self.searched[thread] = self.searched.get(thread, 0) + 1
            self.opened.add(str(args.get("docid", "")))
            return json.dumps(self.retrieval.open(str(args.get("docid", "")), int(args.get("page", 0)))), False
        if name == "done":
            return f"done: {args.get('answer', '')}", True
        return f"unknown tool {name}", False

    async def capture(self, thread: str) -> dict:
        return {"searched": self.searched.get(thread, 0)}
