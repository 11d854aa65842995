"""Analytic prefix-reuse FLOPs of episodes, from their per-request token counts.

    python -m octopus_b200.tools.prefix_flops LOG_DIR [LOG_DIR ...] [--preset qwen2.5-7b] [--lm-head]

For request t of an episode (every thread; requests in log order): P prompt tokens, G
completion tokens, R the prompt tokens an ideal prefix cache serves, U = P - R:
    F_t = C_token (U + G) + C_attn [(P^2 - R^2) / 2 + G P + G^2 / 2]
R follows the append-only cursor protocol: a thread's later request reuses its previous
request's prompt and reply (R = min(P, P_prev + G_prev)); a branch's first request reuses
its parent thread's latest request (R = min(P, P_parent + G_parent)); main's first request
reuses nothing.  The no-reuse figure sets R = 0 everywhere; the report gives both and their
ratio.  A thread that rewinds reuses less, so R is an upper bound there.

Model constants (preset: dense, or hybrid via models.hybrid.hybrid_config):
    C_token = 2 x the non-embedding projection parameters of every layer
    C_attn  = 4 x heads x head_dim x full-attention layers (linear layers have no quadratic term)
--lm-head adds 2 x hidden x vocab per processed token.

Reference parity (behaviour): `scripts/rl_analysis/prefix_flops.py` (the CLM-style analytic
count, the cursor-protocol reuse rule, per-episode and total figures).
"""
from __future__ import annotations

import argparse
import json
from pathlib import Path


def model_constants(preset: str, lm_head: bool = False) -> tuple[float, float]:
    from ..models.config import get_config
    from ..models.hybrid import hybrid_config

    hc = hybrid_config(preset)
    cfg = hc.base if hc is not None else get_config(preset)
    H, F = cfg.hidden, cfg.ffn
    attn_proj = H * cfg.qkv_width + cfg.q_width * H
    mlp = 3 * H * F
    n_attn = sum(1 for i in range(cfg.layers) if hc is None or not hc.is_linear(i))
    n_lin = cfg.layers - n_attn
    lin_proj = (H * 4 * hc.lin_width + H * hc.ba_rows + hc.lin_width * H) if hc is not None else 0
    c_token = 2.0 * (n_attn * (attn_proj + mlp) + n_lin * (lin_proj + mlp))
    if lm_head:
        c_token += 2.0 * H * cfg.vocab_size
    return c_token, 4.0 * cfg.heads * cfg.head_dim * n_attn


def _parent(thread: str) -> str:
    return thread.rsplit("/", 2)[0] if thread.count("/") >= 2 else "main"


def episode_flops(requests: list[dict], c_token: float, c_attn: float) -> dict:
    last: dict[str, tuple[int, int]] = {}
    reuse = none = 0.0
    for r in requests:
        th = str(r.get("thread", "main"))
        P, G = int(r.get("prompt_tokens", 0)), int(r.get("completion_tokens", 0))
        if th in last:
            pp, gp = last[th]
            R = min(P, pp + gp)
        elif th != "main" and _parent(th) in last:
            pp, gp = last[_parent(th)]
            R = min(P, pp + gp)
        else:
            R = 0
        for rr, acc in ((R, "reuse"), (0, "none")):
            f = c_token * (P - rr + G) + c_attn * ((P * P - rr * rr) / 2 + G * P + G * G / 2)
            if acc == "reuse":
                reuse += f
            else:
                none += f
        last[th] = (P, G)
    return {"requests": len(requests), "flops_reuse": reuse, "flops_no_reuse": none,
            "saving": round(1 - reuse / none, 4) if none else None}


def run(log_dirs, preset: str = "qwen2.5-7b", lm_head: bool = False) -> dict:
    c_token, c_attn = model_constants(preset, lm_head)
    eps = []
    for d in log_dirs:
        for f in sorted(Path(d).rglob("requests.jsonl")):
            reqs = [json.loads(x) for x in f.read_text().splitlines() if x.strip()]
            if reqs:
                eps.append({"episode": str(f.parent), **episode_flops(reqs, c_token, c_attn)})
    tot_r = sum(e["flops_reuse"] for e in eps)
    tot_n = sum(e["flops_no_reuse"] for e in eps)
    return {"episodes": len(eps), "flops_reuse": tot_r, "flops_no_reuse": tot_n,
            "saving": round(1 - tot_r / tot_n, 4) if tot_n else None, "per_episode": eps}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m octopus_b200.tools.prefix_flops")
    ap.add_argument("log_dirs", nargs="+")
    ap.add_argument("--preset", default="qwen2.5-7b")
    ap.add_argument("--lm-head", action="store_true")
    args = ap.parse_args(argv)
    res = run(args.log_dirs, args.preset, args.lm_head)
    print(json.dumps({k: v for k, v in res.items() if k != "per_episode"}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
