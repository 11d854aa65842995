"""SWE development evaluation: plan episodes over a task set, graded by the hidden tests.

    python -m octopus_b200.eval.swe_eval --tasks tasks.jsonl [--model-path HF_DIR] [--preset qwen2.5-7b]
        [--samples 1] [--settings episode_settings.json] [--timeout 120] [--bundle 0] [--out results.jsonl]

Tasks: JSONL rows of envs.swe.taskset (instance_id, repo, ref, statement, test_cmd,
hidden_test_cmd, hidden_files).  Each task runs `samples` episodes (main + free forks) on
the in-process engine through the same runtime, chat service and episode switches as
training (`--settings` applies a training run's episode_settings.json), in a fresh copy of
the task's repository; the hidden tests grade the final tree (test-infrastructure edits
undone) and each committed branch's patch alone on its fork point.  Reports the resolve
rate, pass@samples, branch pass rate, completion tokens, requests and critical path.
`--bundle k` evaluates k-task bundles of one repository instead (reward = fraction solved).

Reference parity (behaviour): `octopus/eval/dev_eval.py` (SWE episodes through training's
serving path, eval-equals-train settings, per-episode records and a summary).
"""
from __future__ import annotations

import argparse
import asyncio
import json
import os
import statistics


def _episode_dir(log_dir, spec, s):
    return os.path.join(log_dir, spec.instance_id, str(s)) if log_dir else None


async def run_episodes(svc, specs, samples: int, executor=None, timeout: float = 120.0, max_main_calls=None,
                       log_dir=None):
    from ..envs.swe.taskset import prepare_workspace
    from ..runtime.tree import CursorRuntime

    async def one(spec, s):
        ws = prepare_workspace(spec, executor, timeout)
        rt = CursorRuntime(ws, svc.chat, session_id=f"swe-{spec.instance_id}-{s}", max_main_calls=max_main_calls,
                           log_dir=_episode_dir(log_dir, spec, s))
        res = await rt.run(spec.statement)
        return spec, s, res, ws

    return await asyncio.gather(*[one(t, s) for t in specs for s in range(samples)])


def evaluate(svc, specs, samples: int = 1, executor=None, timeout: float = 120.0, max_main_calls=None,
             engine=None, log_dir=None) -> dict:
    """Per-episode rows and a summary; with log_dir each episode's logs (tree.json, ...) go to
    log_dir/<instance_id>/<sample>/ with its grade in result.json."""
    from ..envs.swe.rl import grade_episode
    from ..rl.group import critical_path
    from ..runtime.core import tree_branches

    results = asyncio.run(run_episodes(svc, specs, samples, executor, timeout, max_main_calls, log_dir))
    rows, by_t = [], {}
    for spec, s, res, ws in results:
        try:
            branches = [br for _, _, br in tree_branches(res["tree"].get("forks") or [])]
            y = grade_episode({"spec": spec}, res["tree"].get("answer"), ws, branches)
        finally:
            ws.discard()
        row = {"instance_id": spec.instance_id, "sample": s, "reward": y, "resolved": y >= 1.0,
               "main_end": res["tree"].get("main_end"), "branches": len(branches),
               "branches_passed": sum(bool(b.get("passed")) for b in branches),
               "completion_tokens": sum(int(r["completion_tokens"]) for r in res["requests"]),
               "requests": len(res["requests"]), "critical_path": critical_path(res["requests"])}
        rows.append(row)
        by_t.setdefault(spec.instance_id, []).append(row["resolved"])
        d = _episode_dir(log_dir, spec, s)
        if d:
            os.makedirs(d, exist_ok=True)
            with open(os.path.join(d, "result.json"), "w") as f:
                json.dump({**row, "reward": y, "task": spec.instance_id}, f)
        if engine is not None:
            for r in res["requests"]:
                if engine.cursors.get(r["id"]) is not None:
                    engine.release_cursor(r["id"])
    nb = sum(r["branches"] for r in rows)
    summary = {"tasks": len(by_t), "episodes": len(rows),
               "resolved": round(statistics.mean(r["resolved"] for r in rows), 4) if rows else 0.0,
               "mean_reward": round(statistics.mean(r["reward"] for r in rows), 4) if rows else 0.0,
               f"pass@{samples}": round(statistics.mean(any(v) for v in by_t.values()), 4) if by_t else 0.0,
               "branch_pass_rate": round(sum(r["branches_passed"] for r in rows) / nb, 4) if nb else None,
               "mean_completion_tokens": round(statistics.mean(r["completion_tokens"] for r in rows), 1) if rows else 0,
               "mean_critical_path": round(statistics.mean(r["critical_path"] for r in rows), 1) if rows else 0}
    return {"summary": summary, "rows": rows}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m octopus_b200.eval.swe_eval")
    ap.add_argument("--tasks", required=True)
    ap.add_argument("--model-path", default="")
    ap.add_argument("--preset", default="qwen2.5-7b")
    ap.add_argument("--samples", type=int, default=1)
    ap.add_argument("--settings", default="")
    ap.add_argument("--timeout", type=float, default=120.0)
    ap.add_argument("--bundle", type=int, default=0)
    ap.add_argument("--max-main-calls", type=int, default=None)
    ap.add_argument("--kv-gb", type=float, default=8.0)
    ap.add_argument("--cpu", action="store_true")
    ap.add_argument("--log-dir", default="", help="per-episode logs (tree.json, result.json) for tree SFT")
    ap.add_argument("--out", default="")
    args = ap.parse_args(argv)

    from ..envs.swe.taskset import build_bundles, load_rows, select_task_specs
    from ..rl.config import run_episode_settings
    from .search_eval import build_service

    if args.settings:
        run_episode_settings(args.settings)
    specs = select_task_specs(load_rows(args.tasks))
    if args.bundle > 1:
        specs = build_bundles(specs, args.bundle)
    svc, eng = build_service(args.preset, args.model_path, args.kv_gb, args.cpu)
    out = evaluate(svc, specs, args.samples, timeout=args.timeout, max_main_calls=args.max_main_calls, engine=eng,
                   log_dir=args.log_dir or None)
    if args.out:
        with open(args.out, "w") as f:
            for r in out["rows"]:
                f.write(json.dumps(r) + "\n")
    print(json.dumps(out["summary"]))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
