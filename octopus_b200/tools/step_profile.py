"""Kernel-time breakdown of one RL step (rollout + train + sync) on one GPU.

    python -m octopus_b200.tools.step_profile [--model qwen2.5-7b] [--instances 32] [--warmup 2]
                                              [--out profile.json]

Runs the bench's single-GPU configuration, then one step under the PyTorch profiler
(CUDA activity trace) and prints the device time per kernel (grouped by name), the
share of each, and the step's phase wall times.  Shares are for finding the next
optimisation; timing numbers come from the CUDA-event bench, not from this run.
"""
from __future__ import annotations

import argparse
import json
import re
from collections import defaultdict


def kernel_group(name: str) -> str:
    n = name
    if "gemm_tcgen05_kernel" in n:
        if "AGather" in n:
            return "ag_gemm (TP all-gather -> GEMM)" + (" split-K" if "EpiSplitK" in n else "")
        if "EpiRS" in n:
            return "gemm_rs (TP GEMM -> reduce-scatter)"
        if "EpiSplitK" in n:
            return "gemm split-K (decode)"
    for pat, g in ((r"gemm_tcgen05_kernel<(\d+), (?:true|false), (?:true|false), octo::EpiHeadLse", "gemm head lse"),
                   (r"gemm_tcgen05_kernel<(\d+), (?:true|false), (?:true|false), octo::EpiHeadGrad", "gemm head grad"),
                   (r"gemm_tcgen05_kernel<(\d+), (?:true|false), (?:true|false), octo::EpiSample", "gemm sample"),
                   (r"gemm_tcgen05_kernel<(\d+), (true|false), (true|false), octo::EpiF32", "gemm f32 (wgrad)"),
                   (r"gemm_tcgen05_kernel<(\d+), (true|false), (true|false), octo::EpiBF16", "gemm bf16"),
                   (r"gemm_tcgen05_kernel", "gemm other")):
        if re.search(pat, n):
            m = re.search(r"gemm_tcgen05_kernel<(\d+), (true|false), (true|false)", n)
            if m and g.startswith("gemm bf16"):
                return f"{g} a_mn={m.group(2)} b_mn={m.group(3)}"
            return g
    m = re.search(r"octo::(\w+)", n)
    if m:
        return m.group(1)
    return n[:80]


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen2.5-7b")
    ap.add_argument("--instances", type=int, default=32)
    ap.add_argument("--samples", type=int, default=4)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--mb-tokens", type=int, default=32768)
    ap.add_argument("--out", default="")
    args = ap.parse_args(argv)

    import torch
    from torch.profiler import ProfilerActivity, profile

    from octopus_b200.envs.dag import DagConfig, MultiAgentDag
    from octopus_b200.models.config import get_config
    from octopus_b200.rl.actor import Actor
    from octopus_b200.rl.trainer import RLTrainer, TrainerConfig
    from octopus_b200.serving.engine import Engine

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = get_config(args.model)
    dcfg = DagConfig(instances=args.instances, samples=args.samples, seed=1000)
    env = MultiAgentDag(cfg.vocab_size, dcfg)
    actor = Actor(cfg, dev, seed=0)
    per_inst = dcfg.prefix_len + dcfg.samples * (4 * (dcfg.turn_len + dcfg.role_len) + 2)
    inst = list(range(args.instances))
    engine = Engine(cfg, actor.weights, kv_slots=int(len(inst) * per_inst * 1.15) + 8192,
                    max_batch=max(8, 1 << (len(inst) * args.samples * 2 - 1).bit_length()), device=dev)

    class _Env:
        def rollout(self, eng):
            return env.rollout(eng, inst)

    tr = RLTrainer(actor, engine, _Env(), TrainerConfig(mb_tokens=args.mb_tokens))
    for _ in range(args.warmup):
        tr.step()
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        st = tr.step()
        torch.cuda.synchronize()
    out = breakdown(prof, st)
    print(json.dumps(out, indent=1))
    if args.out:
        with open(args.out, "w") as f:
            json.dump(out, f, indent=1)


def breakdown(prof, st: dict) -> dict:
    """Device time per kernel group of a profiled step (+ the step's phase wall times)."""
    tot = defaultdict(float)
    cnt = defaultdict(int)
    for e in prof.events():  # noqa: B007
        if e.device_type.name != "CUDA":
            continue
        g = kernel_group(e.name)
        tot[g] += e.device_time_total if hasattr(e, "device_time_total") else e.cuda_time_total
        cnt[g] += 1
    all_us = sum(tot.values())
    rows = sorted(tot.items(), key=lambda kv: -kv[1])
    return {"device_ms_total": round(all_us / 1e3, 1),
            "phases_s": {k: round(st[k], 3) for k in ("rollout_s", "train_s", "sync_s")},
            "kernels": [{"name": k, "ms": round(v / 1e3, 2), "share": round(v / all_us, 4), "launches": cnt[k]}
                        for k, v in rows[:40]]}


if __name__ == "__main__":
    main()
