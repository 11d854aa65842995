"""Rollout-only load on the engine (no trainer, no optimizer step): multi-agent DAG
episodes back to back until N rollouts ran or DURATION seconds passed.  With --switch S,
every S seconds the engine moves to the next weight version (as after a trainer step), so
new requests stop matching KV cached under older versions.  One JSON line per rollout and a
summary line.

    python -m octopus_b200.tools.rollout_load --rollouts 20 --duration 600 [--switch 60]
        [--instances 32 --samples 4 --prefix 2048 --turn 512] [--preset qwen2.5-7b --layers 0]
        [--out rollouts.jsonl]

Reference parity (behaviour): `octopus/tools/rollout_load.py:1-12` (rollout-only load until
N episodes or DURATION, periodic weight-version switches, per-episode records).
"""
from __future__ import annotations

import argparse
import json
import time


def run(engine, env, rollouts: int, duration: float, switch: float = 0.0, out=None) -> dict:
    t_start = time.perf_counter()
    t_switch = t_start
    rows, tokens, versions = [], 0, 0
    for k in range(rollouts):
        if time.perf_counter() - t_start > duration:
            break
        if switch > 0 and k > 0 and time.perf_counter() - t_switch >= switch:
            engine.bump_version()
            versions += 1
            t_switch = time.perf_counter()
        t0 = time.perf_counter()
        ro = env.rollout(engine)
        dt = time.perf_counter() - t0
        row = {"rollout": k, "seconds": round(dt, 4), "generated_tokens": int(ro.generated_tokens),
               "tokens_per_s": round(ro.generated_tokens / dt, 2) if dt > 0 else None,
               "version": int(getattr(engine, "version", 0))}
        rows.append(row)
        tokens += ro.generated_tokens
        if out is not None:
            out.write(json.dumps(row) + "\n")
            out.flush()
    wall = time.perf_counter() - t_start
    return {"rollouts": len(rows), "seconds": round(wall, 3), "generated_tokens": int(tokens),
            "tokens_per_s": round(tokens / wall, 2) if wall > 0 else None, "version_switches": versions}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m octopus_b200.tools.rollout_load")
    ap.add_argument("--rollouts", type=int, default=10)
    ap.add_argument("--duration", type=float, default=600.0)
    ap.add_argument("--switch", type=float, default=0.0, help="seconds between weight-version switches (0: none)")
    ap.add_argument("--instances", type=int, default=32)
    ap.add_argument("--samples", type=int, default=4)
    ap.add_argument("--prefix", type=int, default=2048)
    ap.add_argument("--turn", type=int, default=512)
    ap.add_argument("--preset", default="qwen2.5-7b")
    ap.add_argument("--layers", type=int, default=0)
    ap.add_argument("--kv-slots", type=int, default=0)
    ap.add_argument("--out", default="")
    args = ap.parse_args(argv)

    import torch

    from ..envs.dag import DagConfig, MultiAgentDag
    from ..models.config import get_config
    from ..models.decoder import FlatLayout, Weights, init_flat
    from ..serving.engine import Engine

    dev = torch.device("cuda", 0) if torch.cuda.is_available() else torch.device("cpu")
    cfg = get_config(args.preset, layers=args.layers) if args.layers else get_config(args.preset)
    lay = FlatLayout(cfg)
    w = Weights(cfg, init_flat(cfg, lay, dev, seed=0), lay)
    B = args.instances * args.samples * 2
    slots = args.kv_slots or args.instances * (args.prefix + args.samples * 6 * args.turn) + 4096
    eng = Engine(cfg, w, kv_slots=slots, max_batch=max(8, B), device=dev)
    env = MultiAgentDag(cfg.vocab_size, DagConfig(instances=args.instances, samples=args.samples,
                                                  prefix_len=args.prefix, turn_len=args.turn))
    f = open(args.out, "w") if args.out else None
    try:
        summary = run(eng, env, args.rollouts, args.duration, args.switch, f)
    finally:
        if f is not None:
            f.close()
    print(json.dumps(summary))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
