"""BrowseComp-Plus grading: judged accuracy, the benchmark's retrieval recall and the recall
of the documents the agent opened.

    python -m octopus_b200.eval.bcp run.jsonl --dataset-dir BCP_DIR [--base-url URL/v1] [--model NAME]
        [--workers 16] [--out judged.jsonl]

Run lines: {"query_id", "response", "retrieved_docids", "opened_docids"}, or {"log_dir": DIR,
"query_id"} naming an episode's logs (tree.json + the answer in tree["answer"]), which
`episode_run` converts: main's answer, the docids every thread's searches returned and the
docids it opened, in first-seen order.  Per query, averaged over the run:
  recall            |retrieved & evidence| / |evidence|   (the benchmark's recall)
  open_recall       |opened & evidence| / |evidence|
  open_gold_recall  |opened & gold| / |gold|
An empty response is incorrect without a judge call; a judge failure is counted, not graded.
--out keeps query ids, verdicts, confidences and recalls only: no decoded question or answer
is written.  --base-url / --model default to OCTOPUS_JUDGE_URL / OCTOPUS_JUDGE_MODEL.

Reference parity (behaviour): `octopus/eval/bcp.py:1-106` (run format, episode conversion,
the three recalls, empty responses, judge failures, the redacted output).
"""
from __future__ import annotations

import argparse
import json
import os
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path


def _docids(result: str) -> list[str]:
    """Docids of a search tool result (the workspace returns the retrieval's JSON)."""
    try:
        v = json.loads(result)
    except (json.JSONDecodeError, TypeError):
        return []
    if isinstance(v, dict):
        v = v.get("results", [])
    return [str(r["docid"]) for r in v if isinstance(r, dict) and "docid" in r] if isinstance(v, list) else []


def episode_run(log_dir, query_id) -> dict:
    """A run line from one episode's logs (main and every branch thread)."""
    from ..runtime.core import tree_branches

    tree = json.loads((Path(log_dir) / "tree.json").read_text())
    msgs = list(tree.get("main") or [])
    for _, _, br in tree_branches(tree.get("forks") or []):
        msgs += (br.get("messages") or [])[max(0, int(br.get("prefix_len", 1)) - 1):]
    searches, retrieved, opened = set(), {}, {}
    for m in msgs:
        if m.get("role") == "tool" and m.get("tool_call_id") in searches:
            retrieved.update(dict.fromkeys(_docids(m.get("content") or "")))
        for c in m.get("tool_calls") or []:
            fn = c.get("function") or {}
            if fn.get("name") == "search":
                searches.add(c.get("id"))
            elif fn.get("name") == "open":
                try:
                    args = json.loads(fn.get("arguments") or "{}")
                except ValueError:
                    continue
                opened[str(args.get("docid"))] = None
    return {"query_id": str(query_id), "response": tree.get("answer") or "", "retrieved_docids": list(retrieved),
            "opened_docids": list(opened)}


def _recall(docids, relevant):
    return len(set(docids) & set(relevant)) / len(relevant) if relevant else None


def recalls(line: dict, truth: dict) -> dict:
    opened = line.get("opened_docids", [])
    return {"recall": _recall(line.get("retrieved_docids", []), truth["evidence_docids"]),
            "open_recall": _recall(opened, truth["evidence_docids"]),
            "open_gold_recall": _recall(opened, truth["gold_docids"])}


def evaluate(run: list[dict], truth: dict, judge, workers: int = 16) -> tuple[dict, list[dict]]:
    """judge(question, response, gold) -> (correct | None, confidence | None)."""
    def one(r):
        t = truth[str(r["query_id"])]
        correct, conf = False, None
        if r["response"]:
            try:
                correct, conf = judge(t["query"], r["response"], t["answer"])
            except Exception:  # noqa: BLE001  (an endpoint failure: no verdict, counted)
                correct = None
        return {"query_id": str(r["query_id"]), "correct": correct, "confidence": conf, **recalls(r, t)}

    with ThreadPoolExecutor(max(1, workers)) as pool:
        rows = list(pool.map(one, run))

    def mean(k):
        v = [r[k] for r in rows if r[k] is not None]
        return sum(v) / len(v) if v else None

    return ({"n": len(rows), "accuracy": sum(r["correct"] is True for r in rows) / max(len(rows), 1),
             "judge_failures": sum(r["correct"] is None for r in rows),
             **{k: mean(k) for k in ("recall", "open_recall", "open_gold_recall")}}, rows)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m octopus_b200.eval.bcp")
    ap.add_argument("run")
    ap.add_argument("--dataset-dir", required=True)
    ap.add_argument("--base-url", default=os.environ.get("OCTOPUS_JUDGE_URL", "http://127.0.0.1:30000/v1"))
    ap.add_argument("--model", default=os.environ.get("OCTOPUS_JUDGE_MODEL", "judge"))
    ap.add_argument("--workers", type=int, default=16)
    ap.add_argument("--out", default="")
    a = ap.parse_args(argv)
    from ..envs.search.data import browsecomp_plus
    from ..envs.search.judge import judge as bcp_judge

    key = os.environ.get("OCTOPUS_JUDGE_KEY")
    # no verdict cache here: its keys would hold decoded questions and answers
    judge = lambda q, r, g: bcp_judge(q, r, g, a.base_url, a.model, key, 0.0, None)  # noqa: E731
    lines = [json.loads(x) for x in open(a.run) if x.strip()]
    run = [episode_run(r["log_dir"], r["query_id"]) if "log_dir" in r else r for r in lines if "error" not in r]
    summary, rows = evaluate(run, browsecomp_plus(a.dataset_dir), judge, a.workers)
    if a.out:
        with open(a.out, "w") as f:
            f.writelines(json.dumps(r) + "\n" for r in rows)
    print(json.dumps(summary, indent=1))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
