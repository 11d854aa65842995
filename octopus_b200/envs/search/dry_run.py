"""CPU end-to-end search episode: a fake retrieval corpus and a stub policy served over
HTTP, driven by the real runtime (fork into branches, search, open, done), then graded.

    python -m octopus_b200.envs.search.dry_run

Reference parity (behaviour): `octopus/envs/search/dry_run.py:56-165`.
"""
from __future__ import annotations

import json

from ...runtime.tree import run_episode
from .agent import SearchWorkspace
from .reward import grade
from .service import Retrieval

CORPUS = [
    {"docid": "d1", "title": "Octopus anatomy", "text": "An octopus has three hearts and blue blood. " * 5},
    {"docid": "d2", "title": "Squid facts", "text": "Squids have a beak and eight arms plus two tentacles. " * 5},
    {"docid": "d3", "title": "Cephalopod hearts", "text": "Cephalopods such as the octopus pump blood with three "
                                                          "hearts: two branchial hearts and one systemic heart. " * 5},
]


def call(name, **args):
    return {"id": f"c-{name}", "type": "function", "function": {"name": name, "arguments": json.dumps(args)}}


class StubPolicy:
    """Scripted chat replies per thread: main forks, branches search and answer, main answers."""

    def __init__(self):
        self.step = {}

    def __call__(self, body):
        sid = body["session_id"]
        n = self.step.get(sid, 0)
        self.step[sid] = n + 1
        if sid.endswith("branch-0") or sid.endswith("branch-1"):
            script = [("", [call("search", query="octopus hearts")]), ("", [call("open", docid="d3")]),
                      ("", [call("done", answer="three")])]
        else:
            script = [("", [call("fork", tasks=["count the hearts", "check squids"])]),
                      ("", [call("done", answer="three")])]
        content, calls = script[min(n, len(script) - 1)]
        return {"id": f"{sid}-{n}", "choices": [{"message": {"role": "assistant", "content": content,
                                                             "tool_calls": calls}}],
                "usage": {"prompt_tokens": 100 + 50 * n, "completion_tokens": 20}}


def main():
    ws = SearchWorkspace(Retrieval(CORPUS), "How many hearts does an octopus have?")
    out = run_episode(ws, StubPolicy(), "How many hearts does an octopus have?")
    g = grade(ws.question, out["tree"]["answer"], "3 (three)")
    print(json.dumps({"answer": out["tree"]["answer"], "main_end": out["tree"]["main_end"],
                      "branches": len(out["tree"]["forks"][0]["branches"]) if out["tree"]["forks"] else 0,
                      "grade": g}))
    return out, g


if __name__ == "__main__":
    main()
