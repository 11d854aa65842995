"""Is a mount in the prefix-tree forward the same computation as the engine's mounted
decode (K2 positions)?

    python -m octopus_b200.tools.mount_check [--preset tiny] [--points 8] [--cpu] [--backward]

Per mount point: thread A replies; thread B (its own context) mounts a range of A's
rows and replies.  The engine's behaviour logprobs of B's reply are compared with the
trainer's tree forward of [B's tokens with the mount of A's rows]; without the mount the
same comparison runs on a plain forward.  --backward: a loss on B's reply through the
mounted tree gives finite gradients that reach A's mounted tokens' embeddings.

Reference parity (behaviour): `octopus/tools/mount_check.py` (tree vs K2 cache surgery,
backward through the mount).
"""
from __future__ import annotations

import argparse
import json

import numpy as np


def run(preset="tiny", points=8, device="cpu", backward=False, seed=0):
    import torch

    from ..models.config import get_config
    from ..models.decoder import FlatLayout, Weights, forward_tree, init_flat
    from ..rl.actor import build_microbatch
    from ..rl.workflow import TrainRow, rows_to_microbatches
    from ..serving.engine import Engine, GenInput

    dev = torch.device(device)
    cfg = get_config(preset)
    lay = FlatLayout(cfg)
    grad = torch.zeros(lay.total, dtype=torch.float32, device=dev)
    dtype = torch.float32 if dev.type == "cpu" else torch.bfloat16
    w = Weights(cfg, init_flat(cfg, lay, dev, dtype=dtype, seed=seed, std=0.05), lay, grad)
    eng = Engine(cfg, w, kv_slots=60000, max_batch=16, device=dev, use_graphs=False)
    eng.record_interactions = True
    rng = np.random.default_rng(seed)
    V = cfg.vocab_size
    gaps, gaps_plain, grads = [], [], []
    for p in range(points):
        a = eng.generate([GenInput(rng.integers(1, V, 40 + 5 * p).tolist(), max_new_tokens=12,
                                   cursor_id=f"A{p}")])[0]
        src = eng.cursors.get(f"A{p}")
        s0 = int(rng.integers(0, src.length // 2))
        s1 = int(rng.integers(s0 + 2, src.length - 1))
        for mounted in (True, False):
            cid = f"B{p}{'m' if mounted else ''}"
            b = eng.generate([GenInput(rng.integers(1, V, 20).tolist(), mount=[(f"A{p}", s0, s1)] if mounted else [],
                                       max_new_tokens=8, cursor_id=cid)])[0]
            rec = eng.records[cid]
            toks = rec["tokens"]
            keep = toks >= 0
            n = int(keep.sum())
            mask = np.zeros(n, np.float32)
            mask[-rec["completion"]:] = 1.0
            beh = np.zeros(n, np.float32)
            beh[-rec["completion"]:] = rec["logprobs"]
            row = TrainRow(cid, toks[keep].astype(np.int64), mask, np.ones(n, np.float32), beh,
                           [(0, f"A{p}", s0, s1)] if mounted else [])
            mb = rows_to_microbatches([[row]], eng.records, 1 << 20, lambda *x: build_microbatch(*x, pad_to=8))[0]
            d = mb.to_device(dev)
            grad.zero_()
            with torch.set_grad_enabled(backward and mounted):
                emb = w["embed"]
                lp, _ = forward_tree(w, d.batch, ckpt=False)
                if backward and mounted:
                    lp.float().sum().backward()
                    # the mounted rows' tokens get embedding gradient through the mount
                    src_ids = torch.as_tensor(np.asarray(src.tokens[s0:s1], np.int64), device=dev)
                    g = emb.main_grad.index_select(0, src_ids).norm().item()
                    grads.append(g)
            gap = float((lp.detach().float() - d.behav.float()).abs().max())
            (gaps if mounted else gaps_plain).append(gap)
    out = {"points": points, "mounted_max_gap": max(gaps), "plain_max_gap": max(gaps_plain)}
    if backward:
        out["mounted_token_grad_min"] = min(grads)
        out["grads_finite"] = bool(np.isfinite(grads).all())
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m octopus_b200.tools.mount_check")
    ap.add_argument("--preset", default="tiny")
    ap.add_argument("--points", type=int, default=8)
    ap.add_argument("--backward", action="store_true")
    ap.add_argument("--cpu", action="store_true")
    args = ap.parse_args(argv)
    import torch

    dev = "cpu" if args.cpu or not torch.cuda.is_available() else "cuda"
    print(json.dumps(run(args.preset, args.points, dev, args.backward)))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
