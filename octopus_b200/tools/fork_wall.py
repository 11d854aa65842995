"""Forked episodes against their main-first controls: critical-path cost of the fork tree
(main plus, per fork, its longest branch) against the control's own cost, and the outcome
difference.

    python -m octopus_b200.tools.fork_wall LOG_DIR [LOG_DIR ...] [--unit wall|tokens|calls]

Reads episode logs (tree.json with a "control" record, requests.jsonl with the control's
requests under thread "control", result.json with "reward" and optional "control_reward").
Per pair: C_fork = the fork tree's critical path, C_control = the sum over the control's
requests plus main's requests before its first fork (the control continues that history).
Reports the median C_fork / C_control ratio, the share of pairs where the fork is cheaper,
and, when rewards are present, the mean y - y_control overall, when the fork is cheaper and
when it is not.

Reference parity (behaviour): `scripts/rl_analysis/fork_wall.py` (fork vs main-first control
wall ratio, share where the fork is faster, outcome gain when faster / slower).
"""
from __future__ import annotations

import argparse
import json
import statistics
from pathlib import Path


def _cost(r: dict, unit: str) -> float:
    if unit == "tokens":
        return float(r.get("completion_tokens") or 0)
    if unit == "calls":
        return 1.0
    return float(r.get("elapsed_s") or 0)


def pair(tree: dict, requests: list[dict], unit: str = "wall") -> dict | None:
    from ..rl.group import critical_path

    ctl = tree.get("control")
    if not ctl or "answer" not in ctl:
        return None
    main = [r for r in requests if (r.get("thread") or "main") == "main"]
    before = main[: int(ctl.get("calls_before", 0))]
    c_ctl = sum(_cost(r, unit) for r in before) + sum(_cost(r, unit) for r in requests if r.get("thread") == "control")
    c_fork = critical_path(requests, {"wall": "wall", "tokens": "tokens", "calls": "calls"}[unit])
    return {"c_fork": c_fork, "c_control": c_ctl, "ratio": c_fork / c_ctl if c_ctl else None}


def run(log_dirs, unit: str = "wall") -> dict:
    rows = []
    for d in log_dirs:
        for tf in sorted(Path(d).rglob("tree.json")):
            rq = tf.parent / "requests.jsonl"
            if not rq.exists():
                continue
            p = pair(json.loads(tf.read_text()), [json.loads(x) for x in rq.read_text().splitlines() if x.strip()],
                     unit)
            if p is None or p["ratio"] is None:
                continue
            res = tf.parent / "result.json"
            if res.exists():
                r = json.loads(res.read_text())
                if r.get("reward") is not None and r.get("control_reward") is not None:
                    p["gain"] = float(r["reward"]) - float(r["control_reward"])
            rows.append(p)
    if not rows:
        return {"pairs": 0}
    faster = [p for p in rows if p["ratio"] < 1]
    out = {"pairs": len(rows), "ratio_median": round(statistics.median(p["ratio"] for p in rows), 4),
           "fork_cheaper": round(len(faster) / len(rows), 4)}
    g = [p for p in rows if "gain" in p]
    if g:
        mean = lambda xs: round(statistics.mean(xs), 4) if xs else None  # noqa: E731
        out.update({"gain": mean([p["gain"] for p in g]), "gain_when_cheaper": mean([p["gain"] for p in g
                                                                                      if p["ratio"] < 1]),
                    "gain_when_not": mean([p["gain"] for p in g if p["ratio"] >= 1])})
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m octopus_b200.tools.fork_wall")
    ap.add_argument("log_dirs", nargs="+")
    ap.add_argument("--unit", choices=("wall", "tokens", "calls"), default="wall")
    args = ap.parse_args(argv)
    print(json.dumps(run(args.log_dirs, args.unit)))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
