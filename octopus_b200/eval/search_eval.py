"""Search evaluation: agent-runtime episodes over a question set, graded.

    python -m octopus_b200.eval.search_eval --questions q.jsonl --corpus corpus.jsonl
        [--model-path HF_DIR] [--preset qwen2.5-7b] [--samples 1] [--settings episode_settings.json]
        [--judge-url http://host:port/v1 --judge-model NAME] [--out results.jsonl]

Questions: JSONL {qid, question, answer[, evidence: [docid, ...]]}; corpus: JSONL
{docid, title, text}.  Each question runs `samples` episodes on the in-process engine
(the same runtime, chat service and episode switches as training: `--settings` applies
a training run's episode_settings.json so evaluation runs the episodes training saw).
Reports accuracy (exact match, else the judge when given), pass@samples, evidence
recall (an evidence document was opened), completion tokens, requests and the critical
path (longest dependent chain of completion tokens) per episode.

Reference parity (behaviour): `octopus/eval/search_dev_eval.py`, `octopus/eval/bcp.py`
(judged accuracy and recall), eval-equals-train settings (`octopus/rl/config.py`).
"""
from __future__ import annotations

import argparse
import asyncio
import json
import statistics


def judge_via_http(url: str, model: str = "judge", key: str | None = None, temperature: float = 0.0,
                   cache: str | None = None):
    """judge(question, response, gold) -> bool | None: the BrowseComp-Plus grader
    (envs.search.judge) on an OpenAI-compatible endpoint (base URL ending in /v1)."""
    from ..envs.search.judge import judge as bcp_judge

    def judge(question, response, gold):
        return bcp_judge(question, response, gold, url, model, key, temperature, cache)[0]

    return judge


async def run_episodes(svc, retrieval, questions, samples: int, max_main_calls=None):
    from ..envs.search.agent import SearchWorkspace
    from ..runtime.tree import CursorRuntime

    async def one(q, s):
        ws = SearchWorkspace(retrieval, q["question"])
        rt = CursorRuntime(ws, svc.chat, session_id=f"eval-{q['qid']}-{s}", max_main_calls=max_main_calls)
        res = await rt.run(q["question"])
        return q, s, res, ws

    return await asyncio.gather(*[one(q, s) for q in questions for s in range(samples)])


def evaluate(svc, retrieval, questions, samples: int = 1, judge=None, max_main_calls=None, engine=None) -> dict:
    from ..envs.search.reward import grade
    from ..rl.group import critical_path

    results = asyncio.run(run_episodes(svc, retrieval, questions, samples, max_main_calls))
    rows, by_q = [], {}
    for q, s, res, ws in results:
        ans = res["tree"].get("answer")
        g = grade(q["question"], ans, q["answer"], judge)
        ev = set(q.get("evidence") or [])
        row = {"qid": q["qid"], "sample": s, "answer": ans, "correct": g["correct"], "by": g["by"],
               "recall": (len(ev & ws.opened) > 0) if ev else None,
               "completion_tokens": sum(int(r["completion_tokens"]) for r in res["requests"]),
               "requests": len(res["requests"]), "critical_path": critical_path(res["requests"]),
               "branches": sum(len(f.get("branches") or []) for f in res["tree"].get("forks") or [])}
        rows.append(row)
        by_q.setdefault(q["qid"], []).append(row["correct"])
        if engine is not None:
            for r in res["requests"]:
                if engine.cursors.get(r["id"]) is not None:
                    engine.release_cursor(r["id"])
    rec = [r["recall"] for r in rows if r["recall"] is not None]
    summary = {"questions": len(by_q), "episodes": len(rows),
               "accuracy": round(statistics.mean(r["correct"] for r in rows), 4) if rows else 0.0,
               f"pass@{samples}": round(statistics.mean(any(v) for v in by_q.values()), 4) if by_q else 0.0,
               "recall": round(statistics.mean(rec), 4) if rec else None,
               "mean_completion_tokens": round(statistics.mean(r["completion_tokens"] for r in rows), 1) if rows else 0,
               "mean_critical_path": round(statistics.mean(r["critical_path"] for r in rows), 1) if rows else 0}
    return {"summary": summary, "rows": rows}


def build_service(preset: str, model_path: str = "", kv_gb: float = 8.0, cpu: bool = False):
    """(ChatService, Engine) on cuda:0 (CPU with `cpu` or without a GPU): Hugging Face
    weights from `model_path`, else random-init weights of `preset` with the tiny tokenizer."""
    import torch

    from ..models.config import get_config
    from ..models.decoder import FlatLayout, Weights, init_flat, load_hf
    from ..serving.chat import ChatTokenizer
    from ..serving.engine import Engine
    from ..serving.local import ChatService

    dev = torch.device("cpu") if cpu or not torch.cuda.is_available() else torch.device("cuda", 0)
    tok = ChatTokenizer.from_dir(model_path) if model_path else ChatTokenizer.tiny()
    cfg = get_config(preset)
    if not model_path and cfg.vocab_size < tok.vocab_size:
        cfg = cfg.with_(vocab_size=(tok.vocab_size + 127) // 128 * 128)
    lay = FlatLayout(cfg)
    w = Weights(cfg, init_flat(cfg, lay, dev, dtype=torch.bfloat16 if dev.type == "cuda" else torch.float32), lay)
    if model_path:
        load_hf(w, model_path)
    kv_slots = int(kv_gb * (1 << 30) / (4 * cfg.layers * cfg.kv_width))
    eng = Engine(cfg, w, kv_slots=kv_slots, max_batch=64, device=dev)
    return ChatService(eng, tok), eng


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m octopus_b200.eval.search_eval")
    ap.add_argument("--questions", required=True)
    ap.add_argument("--corpus", required=True)
    ap.add_argument("--model-path", default="")
    ap.add_argument("--preset", default="qwen2.5-7b")
    ap.add_argument("--samples", type=int, default=1)
    ap.add_argument("--settings", default="")
    ap.add_argument("--judge-url", default="")
    ap.add_argument("--judge-model", default="judge")
    ap.add_argument("--max-main-calls", type=int, default=None)
    ap.add_argument("--kv-gb", type=float, default=8.0)
    ap.add_argument("--cpu", action="store_true")
    ap.add_argument("--out", default="")
    args = ap.parse_args(argv)

    from ..envs.search.agent import search_defaults
    from ..envs.search.service import Retrieval
    from ..rl.config import run_episode_settings

    if args.settings:
        run_episode_settings(args.settings)
    search_defaults()
    svc, eng = build_service(args.preset, args.model_path, args.kv_gb, args.cpu)
    questions = [json.loads(x) for x in open(args.questions) if x.strip()]
    corpus = [json.loads(x) for x in open(args.corpus) if x.strip()]
    judge = judge_via_http(args.judge_url, args.judge_model) if args.judge_url else None
    res = evaluate(svc, Retrieval(corpus), questions, args.samples, judge, args.max_main_calls, eng)
    print(json.dumps(res["summary"]))
    if args.out:
        with open(args.out, "w") as f:
            for r in res["rows"]:
                f.write(json.dumps(r) + "\n")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
