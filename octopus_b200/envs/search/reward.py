"""Search answers: normalised exact match (SQuAD-style normalisation, numbers must match
as written), else an optional judge callable; the episode outcome and group credit
with the search gate (a branch keeps its advantage only if it closed with done, a
non-empty summary, and searched at least once).

Reference parity (behaviour): `octopus/envs/search/reward.py:58-206`.
"""
from __future__ import annotations

import re
import string

from ...rl.group import group_step, search_gate


def normalize(text: str) -> str:
    text = re.sub(r"\\(?:boxed|text)\s*\{", "", str(text))
    text = "".join(ch for ch in text.lower() if ch not in string.punctuation)
    return " ".join(w for w in text.split() if w not in ("a", "an", "the"))


def numbers(text: str) -> list[str]:
    return re.findall(r"-?\d+(?:[.,:/]\d+)*", str(text))


def exact_match(response: str, gold: str) -> bool:
    return normalize(response) == normalize(gold) != "" and numbers(response) == numbers(gold)


def grade(question: str, response: str, gold: str, judge=None) -> dict:
    """{correct, by}: exact match first, then judge(question, response, gold) -> bool | None
    (given, else the BrowseComp-Plus judge configured by OCTOPUS_JUDGE_*: envs.search.judge);
    a judge without a verdict grades incorrect ("judge_unparsed")."""
    if response is None or not str(response).strip():
        return {"correct": False, "by": "empty"}
    if exact_match(response, gold):
        return {"correct": True, "by": "exact"}
    if judge is None:
        from .judge import env_judge

        judge = env_judge()
    if judge is not None:
        v = judge(question, response, gold)
        return {"correct": False, "by": "judge_unparsed"} if v is None else {"correct": bool(v), "by": "judge"}
    return {"correct": False, "by": "exact"}


def search_outcome(answer: str | None, gold: str, question: str = "", judge=None) -> float:
    return 1.0 if grade(question, answer, gold, judge)["correct"] else 0.0


def search_group_step(episodes: list[dict], branch_credit: str = "gate") -> list[dict]:
    return group_step(episodes, branch_credit, gate=search_gate if branch_credit == "gate" else None)
