"""Rollout-only evaluation of the synthetic multi-agent DAG (no training): rewards,
generated tokens, cache reuse and throughput of the rollout engine.

    python -m octopus_b200.eval.dag_eval [--preset qwen2.5-7b] [--instances 32] [--samples 4] [--steps 2]

Reference parity (behaviour): the rollout half of `octopus/eval/dev_eval.py` (episodes
through the training stack, no update) on this framework's synthetic DAG workload.
"""
from __future__ import annotations

import argparse
import json
import time


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m octopus_b200.eval.dag_eval")
    ap.add_argument("--preset", default="qwen2.5-7b")
    ap.add_argument("--layers", type=int, default=0)
    ap.add_argument("--instances", type=int, default=32)
    ap.add_argument("--samples", type=int, default=4)
    ap.add_argument("--prefix", type=int, default=2048)
    ap.add_argument("--turn", type=int, default=512)
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--cpu", action="store_true")
    args = ap.parse_args(argv)

    import torch

    from ..envs.dag import DagConfig, MultiAgentDag
    from ..models.config import get_config
    from ..models.decoder import FlatLayout, Weights, init_flat
    from ..serving.engine import Engine

    dev = torch.device("cpu") if args.cpu or not torch.cuda.is_available() else torch.device("cuda", 0)
    cfg = get_config(args.preset, **({"layers": args.layers} if args.layers else {}))
    lay = FlatLayout(cfg)
    w = Weights(cfg, init_flat(cfg, lay, dev, dtype=torch.bfloat16 if dev.type == "cuda" else torch.float32), lay)
    dcfg = DagConfig(instances=args.instances, samples=args.samples, prefix_len=args.prefix, turn_len=args.turn)
    per = dcfg.prefix_len + dcfg.samples * (4 * (dcfg.turn_len + dcfg.role_len) + 2)
    eng = Engine(cfg, w, kv_slots=int(args.instances * per * 1.15) + 4096,
                 max_batch=max(8, 1 << (args.instances * args.samples * 2 - 1).bit_length()), device=dev)
    env = MultiAgentDag(cfg.vocab_size, dcfg)
    for step in range(args.steps):
        s0 = dict(eng.stats)
        t0 = time.perf_counter()
        ro = env.rollout(eng)
        if dev.type == "cuda":
            torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        d = {k: eng.stats[k] - s0[k] for k in ("prefill_tokens", "cached_tokens", "decode_steps")}
        print(json.dumps({"step": step + 1, "seconds": round(dt, 3), "generated_tokens": ro.generated_tokens,
                          "tokens_per_s": round(ro.generated_tokens / dt, 1),
                          "mean_reward": sum(ro.rewards) / len(ro.rewards), **d,
                          "cache_reuse": round(d["cached_tokens"] / max(1, d["cached_tokens"] + d["prefill_tokens"]),
                                               4)}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
