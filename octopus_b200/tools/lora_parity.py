"""Do the rollout engine (merged W + s B A) and the trainer (base + adapter, unmerged)
score the same tokens alike, with an adapter on every target?

    python -m octopus_b200.tools.lora_parity [--preset tiny] [--rank 8] [--randomize] [--cpu]

A random adapter (B != 0, --randomize) makes a projection the engine misses show up: the
gap then grows to the size of the adapter's effect instead of staying at the numeric
noise floor of the base.  Reports the max |logp gap| with and without the adapter.

Reference parity (behaviour): `octopus/tools/lora_parity.py` (server vs trainer logprobs,
randomized adapter so a skipped module shows).
"""
from __future__ import annotations

import argparse
import json

import numpy as np


def run(preset="tiny", rank=8, randomize=True, device="cpu", seed=0, n_tokens=48):
    import torch

    from ..models.config import get_config
    from ..models.decoder import forward_tree
    from ..models.lora import LoRAConfig
    from ..rl.actor import LoRAActor, build_microbatch
    from ..serving.engine import Engine, GenInput

    dev = torch.device(device)
    cfg = get_config(preset)
    dt = torch.float32 if dev.type == "cpu" else torch.bfloat16
    act = LoRAActor(cfg, dev, lora=LoRAConfig(rank, 2.0 * rank), dtype=dt, ckpt=False, seed=seed)
    if randomize:
        g = torch.Generator(device="cpu").manual_seed(seed + 5)
        for name, t in act.lora.t.items():
            if name.endswith(".B"):
                t.copy_((torch.randn(t.shape, generator=g) * 0.02).to(t.dtype))
        act.lora.master.copy_(act.lora.flat16.to(act.lora.master.dtype))
        act.optimizer_merge()
    eng = Engine(cfg, act.serving, kv_slots=20000, max_batch=8, device=dev, use_graphs=False)
    rng = np.random.default_rng(seed)
    prompt = rng.integers(1, cfg.vocab_size, n_tokens).tolist()
    out = eng.generate([GenInput(prompt, max_new_tokens=8)])[0]
    full = np.asarray(prompt + out.output_ids)
    n = len(full)
    mask = np.r_[np.zeros(n - 8), np.ones(8)].astype(np.float32)
    mb = build_microbatch(full, [0, n], None, mask, np.zeros(n, np.float32), np.zeros(n, np.float32), pad_to=8)
    d = mb.to_device(dev)
    with torch.no_grad():
        lp_lora, _ = forward_tree(act.base, d.batch, ckpt=False, lora=act.lora)
        lp_base, _ = forward_tree(act.base, d.batch, ckpt=False)
    eng_lp = torch.as_tensor(out.output_logprobs, dtype=torch.float32)
    return {"engine_vs_trainer_lora": float((lp_lora.float().cpu() - eng_lp).abs().max()),
            "engine_vs_trainer_base": float((lp_base.float().cpu() - eng_lp).abs().max()),
            "randomized": randomize}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m octopus_b200.tools.lora_parity")
    ap.add_argument("--preset", default="tiny")
    ap.add_argument("--rank", type=int, default=8)
    ap.add_argument("--randomize", action="store_true")
    ap.add_argument("--cpu", action="store_true")
    args = ap.parse_args(argv)
    import torch

    dev = "cpu" if args.cpu or not torch.cuda.is_available() else "cuda"
    print(json.dumps(run(args.preset, args.rank, args.randomize, dev)))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
