"""Trainer memory bench: one actor forward + backward on a synthetic prefix-tree micro-batch
under several memory settings, each reporting the GPU peak, the pinned host bytes of saved
activations, the time, and the relative L2 distance of its gradients to the first
setting's (list a setting twice for the run-to-run noise floor).

    python -m octopus_b200.tools.act_gpu_bench --tokens 65536 --settings layer host:0 host:8 chunk:32768 \\
        tile:16384 block:2 [--preset qwen2.5-7b] [--layers 0] [--lora 0] [--group 8]

Settings: `layer` (per-layer checkpoint), `block:K` (every K-th layer input kept),
`host:GB` (saved activations past GB of GPU memory go to pinned host memory), `chunk:N`
(chunk-major, chunks of N tree rows), `tile:N` (o-projection + MLP in checkpointed tiles of
N rows); `+` combines them (`chunk:32768+tile:8192`).  The micro-batch is a GRPO-like group:
--group sequences sharing a prefix of a sixth of the tree.

Reference parity (behaviour): `octopus/tools/act_gpu_bench.py:1-8` (a forward + backward per
ACT_GPU_GB value: GPU peak, pinned host bytes, time, gradient distance to the first).
"""
from __future__ import annotations

import argparse
import json
import time

import numpy as np


def group_tree(tree_tokens: int, n: int, vocab: int, seed: int = 0):
    """n sequences sharing a prefix of a sixth of the tree (flat tokens, cu)."""
    rng = np.random.default_rng(seed)
    prefix = rng.integers(1, vocab, max(1, tree_tokens // 6))
    own = max(1, (tree_tokens - len(prefix)) // n)
    seqs = [np.r_[prefix, rng.integers(1, vocab, own)] for _ in range(n)]
    flat = np.concatenate(seqs)
    return flat, np.r_[0, np.cumsum([len(s) for s in seqs])]


def parse_setting(s: str) -> dict:
    kw = {"ckpt_block": 1, "act_gpu_bytes": None, "chunk_tokens": 0, "seq_tile": 0}
    for part in s.split("+"):
        name, _, val = part.partition(":")
        if name == "layer":
            continue
        if name == "block":
            kw["ckpt_block"] = int(val)
        elif name == "host":
            kw["act_gpu_bytes"] = int(float(val) * (1 << 30))
        elif name == "chunk":
            kw["chunk_tokens"] = int(val)
        elif name == "tile":
            kw["seq_tile"] = int(val)
        else:
            raise ValueError(f"unknown setting {part!r}")
    return kw


def run(settings, tokens: int, preset: str = "qwen2.5-7b", layers: int = 0, lora: int = 0, group: int = 8,
        device=None, dtype=None) -> list[dict]:
    import torch

    from ..models.config import get_config
    from ..rl.actor import Actor, LoRAActor, build_microbatch

    dev = torch.device(device) if device is not None else (
        torch.device("cuda", 0) if torch.cuda.is_available() else torch.device("cpu"))
    cfg = get_config(preset, layers=layers) if layers else get_config(preset)
    dtype = dtype or (torch.bfloat16 if dev.type == "cuda" else torch.float64)
    if lora:
        from ..models.lora import LoRAConfig

        actor = LoRAActor(cfg, dev, lora=LoRAConfig(r=lora, alpha=lora), seed=0, dtype=dtype)
    else:
        actor = Actor(cfg, dev, seed=0, dtype=dtype)
    flat, cu = group_tree(tokens, group, cfg.vocab_size)
    n = len(flat)
    rng = np.random.default_rng(1)
    mb = build_microbatch(flat, cu, None, np.ones(n, np.float32), rng.normal(size=n).astype(np.float32),
                          np.zeros(n, np.float32), pad_to=128 if dev.type == "cuda" else 8)
    out, ref = [], None
    for s in settings:
        kw = parse_setting(s)
        actor.set_memory(**kw)
        actor.zero_grad()
        if dev.type == "cuda":
            torch.cuda.synchronize()
            torch.cuda.reset_peak_memory_stats(dev)
        t0 = time.perf_counter()
        actor.forward_backward([mb])
        if dev.type == "cuda":
            torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        g = actor.grad.double().clone()
        rel = 0.0 if ref is None else float((g - ref).norm() / (ref.norm() + 1e-30))
        ref = g if ref is None else ref
        host = actor.host_acts
        out.append({"setting": s, "tree_tokens": int(mb.n_tree), "seconds": round(dt, 4),
                    "gpu_peak_gb": round(torch.cuda.max_memory_allocated(dev) / 2 ** 30, 3) if dev.type == "cuda"
                    else None,
                    "host_gb": round(host.host_bytes / 2 ** 30, 3) if host is not None else 0.0,
                    "grad_rel_l2": rel})
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m octopus_b200.tools.act_gpu_bench")
    ap.add_argument("--tokens", type=int, nargs="+", default=[65536])
    ap.add_argument("--settings", nargs="+", default=["layer", "layer", "host:0", "chunk:32768", "tile:16384"])
    ap.add_argument("--preset", default="qwen2.5-7b")
    ap.add_argument("--layers", type=int, default=0)
    ap.add_argument("--lora", type=int, default=0, help="LoRA rank (0: full fine-tuning)")
    ap.add_argument("--group", type=int, default=8)
    ap.add_argument("--cpu", action="store_true")
    args = ap.parse_args(argv)
    for t in args.tokens:
        for row in run(args.settings, t, args.preset, args.layers, args.lora, args.group,
                       device="cpu" if args.cpu else None):
            print(json.dumps(row), flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
