"""Training-side bench on synthetic trees: forward + backward of the actor on one micro-
batch per requested shape, with peak memory and speed.

    python -m octopus_b200.tools.replay_bench --synthetic 65536 131072 [--branch 40000:20000 ...]
        [--preset qwen2.5-7b] [--layers 0] [--ckpt-block 1] [--act-gpu-gb -1]

Each micro-batch is one thread of the given length plus one branch per --branch
SHARED:OWN (its first SHARED tokens shared with the thread, then OWN new tokens), built
into a prefix tree; every token is scored.

Reference parity (behaviour): `octopus/tools/replay_bench.py` (--synthetic lengths and
--branch SHARED:OWN, peak memory and speed of the actor's forward + backward).
"""
from __future__ import annotations

import argparse
import json
import time

import numpy as np


def make_tree(length: int, branches, vocab: int, seed: int = 0):
    rng = np.random.default_rng(seed)
    main = rng.integers(1, vocab, length)
    seqs = [main]
    for shared, own in branches:
        seqs.append(np.r_[main[:shared], rng.integers(1, vocab, own)])
    flat = np.concatenate(seqs)
    cu = np.r_[0, np.cumsum([len(s) for s in seqs])]
    return flat, cu


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m octopus_b200.tools.replay_bench")
    ap.add_argument("--synthetic", type=int, nargs="+", required=True)
    ap.add_argument("--branch", nargs="*", default=[])
    ap.add_argument("--preset", default="qwen2.5-7b")
    ap.add_argument("--layers", type=int, default=0)
    ap.add_argument("--ckpt-block", type=int, default=1)
    ap.add_argument("--act-gpu-gb", type=float, default=-1.0)
    ap.add_argument("--cpu", action="store_true")
    args = ap.parse_args(argv)

    import torch

    from ..models.config import get_config
    from ..rl.actor import Actor, build_microbatch

    dev = torch.device("cpu") if args.cpu or not torch.cuda.is_available() else torch.device("cuda", 0)
    cfg = get_config(args.preset, **({"layers": args.layers} if args.layers else {}))
    actor = Actor(cfg, dev, seed=0, dtype=torch.bfloat16 if dev.type == "cuda" else torch.float32)
    actor.set_memory(args.ckpt_block, int(args.act_gpu_gb * (1 << 30)) if args.act_gpu_gb >= 0 else None)
    br = [tuple(int(x) for x in b.split(":")) for b in args.branch]
    for L in args.synthetic:
        flat, cu = make_tree(L, br, cfg.vocab_size)
        n = len(flat)
        mb = build_microbatch(flat, cu, None, np.ones(n, np.float32), np.random.default_rng(1).normal(size=n)
                              .astype(np.float32), np.zeros(n, np.float32))
        if dev.type == "cuda":
            torch.cuda.synchronize()
            torch.cuda.reset_peak_memory_stats(dev)
        t0 = time.perf_counter()
        actor.zero_grad()
        actor.forward_backward([mb])
        if dev.type == "cuda":
            torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        peak = torch.cuda.max_memory_allocated(dev) / 2**30 if dev.type == "cuda" else None
        host = actor.host_acts.host_bytes / 2**30 if actor.host_acts is not None else 0.0
        print(json.dumps({"flat_tokens": int(n), "tree_tokens": int(mb.n_tree), "seconds": round(dt, 3),
                          "tree_tokens_per_s": round(mb.n_tree / dt, 1), "gpu_peak_gib": peak,
                          "host_act_gib": round(host, 3)}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
