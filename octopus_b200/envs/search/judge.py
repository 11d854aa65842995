"""BrowseComp-Plus judge: the benchmark's grader prompt and reply parser on any
OpenAI-compatible chat endpoint, shared by training rewards and evaluation.

  judge(question, response, gold, url, model, key, temperature) -> (correct | None, confidence | None)
  parse_judge(text) -> (correct, confidence): "**correct:** yes", "**correct**: yes" or
                       "correct: yes" (first form found), the confidence likewise (capped at 100)
  env_judge() -> judge(question, response, gold) -> bool | None from the environment:
                 OCTOPUS_JUDGE_URL (base URL ending in /v1; unset: no judge),
                 OCTOPUS_JUDGE_MODEL ("judge"), OCTOPUS_JUDGE_KEY (bearer, optional),
                 OCTOPUS_JUDGE_TEMPERATURE (0), OCTOPUS_JUDGE_TIMEOUT (600 s),
                 OCTOPUS_JUDGE_CACHE (JSONL of past verdicts; unset: none)

A reply without a verdict gets one follow-up on the same conversation asking for the two
lines alone; still none: correct is None (graded incorrect, counted as unparsed).  An
endpoint failure raises (after the transport's retries): an episode whose grade failed is
an error, never a training signal.  The cache is keyed on the endpoint's model identity
(`/model_info` model_path when the server gives one, else the served name), the temperature
and the three texts; only verdicts are cached, one short line per append.  Request settings
follow the benchmark's evaluation script: top_p 0.8, top_k 20, 4096 tokens, thinking off.

Reference parity (behaviour): `octopus/envs/search/reward.py:1-186` (grader prompt, parser
forms, follow-up, cache keyed on judge identity, environment settings); the grader text is
BrowseComp-Plus's published `scripts_evaluation/evaluate_run.py` template, kept word for
word so judged accuracy is comparable with the benchmark's.
"""
from __future__ import annotations

import functools
import json
import os
import re
import threading
import urllib.request

GRADER_TEMPLATE = """
Judge whether the following [response] to [question] is correct or not based on the precise and unambiguous [correct_answer] below.

[question]: {question}

[response]: {response}

[correct_answer]: {correct_answer}

Your judgement must be in the format and criteria specified below:

extracted_final_answer: The final exact answer extracted from the [response].

[correct_answer]: Repeat the [correct_answer] given above.

reasoning: Explain why the extracted_final_answer is correct or incorrect based on [correct_answer], in the context of this [question]. You should judge whether the extracted_final_answer is semantically equivalent to [correct_answer], allowing the extracted_final_answer to be string variations of [correct_answer]. You should also allow the extracted_final_answer to be more precise or verbose than [correct_answer], as long as its additional details are correct. Do not comment on any background to the problem, do not attempt to solve the problem, do not argue for any answer different than [correct_answer], focus only on whether the answers are semantically equivalent.

correct: Answer 'yes' if extracted_final_answer matches the [correct_answer] given above, or is within a small margin of error for numerical problems. Answer 'no' otherwise, i.e. if there if there is any inconsistency, ambiguity, non-equivalency, or if the extracted answer is incorrect.


confidence: The extracted confidence score between 0|\\%| and 100|\\%| from [response]. Put 100 if there is no confidence score available.
""".strip()  # noqa: E501

FOLLOW_UP = "State your judgement as two lines only:\ncorrect: yes or no\nconfidence: a number from 0 to 100"

_lock = threading.Lock()


def parse_judge(text: str) -> tuple[bool | None, float | None]:
    def field(name: str, value: str):
        for pat in (rf"\*\*{name}:\*\*\s*{value}", rf"\*\*{name}\*\*:\s*{value}", rf"{name}:\s*{value}"):
            m = re.search(pat, text, re.I)
            if m:
                return m.group(1)
        return None

    c, conf = field("correct", "(yes|no)"), field("confidence", r"(\d+(?:\.\d+)?)")
    return (c.lower() == "yes" if c else None), (min(float(conf), 100.0) if conf else None)


@functools.lru_cache(maxsize=64)
def judge_identity(url: str, model: str, key: str | None = None) -> str:
    """The model behind the endpoint's served name: its /model_info model_path when the server
    reports one for `model`, else the served name itself."""
    info_url = url.rstrip("/").removesuffix("/v1") + "/model_info"
    headers = {"Authorization": "Bearer " + key} if key else {}
    try:
        with urllib.request.urlopen(urllib.request.Request(info_url, headers=headers), timeout=60) as r:
            info = json.load(r)
    except (OSError, ValueError):
        return model
    if info.get("served_model_name") in (None, model) and info.get("model_path"):
        return str(info["model_path"])
    return model


def _post(url, body, headers, timeout):
    from ...runtime.core import post_chat

    return post_chat(url.rstrip("/") + "/chat/completions", body, headers, timeout=timeout)


def judge(question: str, response: str, gold: str, url: str, model: str = "judge", key: str | None = None,
          temperature: float = 0.0, cache: str | None = None, post=None) -> tuple[bool | None, float | None]:
    post = post or _post
    ck = None
    if cache:
        ck = ["bcp", judge_identity(url, model, key), temperature, question, response, gold]
        if os.path.exists(cache):
            with open(cache) as f:
                for line in f:
                    row = json.loads(line)
                    if row.get("key") == ck:
                        return row["correct"], row["confidence"]
    body = {"model": model, "temperature": temperature, "top_p": 0.8, "top_k": 20, "max_tokens": 4096,
            "chat_template_kwargs": {"enable_thinking": False},
            "messages": [{"role": "user", "content": GRADER_TEMPLATE.format(question=question, response=response,
                                                                            correct_answer=gold)}]}
    headers = {"Content-Type": "application/json", **({"Authorization": "Bearer " + key} if key else {})}
    timeout = int(os.environ.get("OCTOPUS_JUDGE_TIMEOUT", "600"))

    def ask() -> str:
        out = post(url, body, headers, timeout)
        return out["choices"][0]["message"].get("content") or ""

    reply = ask()
    correct, conf = parse_judge(reply)
    if correct is None:
        body["messages"] += [{"role": "assistant", "content": reply}, {"role": "user", "content": FOLLOW_UP}]
        correct, conf = parse_judge(ask())
    if correct is not None and cache:
        with _lock, open(cache, "a") as f:
            f.write(json.dumps({"key": ck, "correct": correct, "confidence": conf}) + "\n")
    return correct, conf


def env_judge():
    """A judge(question, response, gold) -> bool | None configured by OCTOPUS_JUDGE_*, or None
    when OCTOPUS_JUDGE_URL is unset."""
    url = os.environ.get("OCTOPUS_JUDGE_URL")
    if not url:
        return None
    model = os.environ.get("OCTOPUS_JUDGE_MODEL", "judge")
    key = os.environ.get("OCTOPUS_JUDGE_KEY")
    temp = float(os.environ.get("OCTOPUS_JUDGE_TEMPERATURE", "0"))
    cache = os.environ.get("OCTOPUS_JUDGE_CACHE")

    def j(question, response, gold):
        return judge(question, response, gold, url, model, key, temp, cache)[0]

    return j


__all__ = ["FOLLOW_UP", "GRADER_TEMPLATE", "env_judge", "judge", "judge_identity", "parse_judge"]
