"""Is the prefix-tree forward the same computation as running each sequence alone?

    python -m octopus_b200.tools.tree_check [--preset tiny] [--n-seqs 4] [--prefix 300] [--tail 200]
                                            [--layers 0] [--cpu] [--seed 0]

Random sequences sharing a prefix are scored at every position three ways: each
sequence alone, the ordinary packed varlen batch (no prefix sharing), and the prefix
tree.  Reports the logprob gaps (tree vs alone, packed vs alone: the packed gap is the
numeric noise floor the tree has to match) and the relative L2 distance of the weight
gradients of one weighted loss (tree vs packed).

Reference parity (behaviour): `octopus/tools/tree_check.py` (alone / packed / tree, logprobs
and gradients of one weighted loss).
"""
from __future__ import annotations

import argparse
import json

import numpy as np


def run(preset="tiny", n_seqs=4, prefix=300, tail=200, layers=0, device="cpu", seed=0):
    import torch

    from ..models.config import get_config
    from ..models.decoder import FlatLayout, Weights, forward_tree, init_flat
    from ..rl.actor import build_microbatch

    dev = torch.device(device)
    cfg = get_config(preset, **({"layers": layers} if layers else {}))
    lay = FlatLayout(cfg)
    dtype = torch.float32 if dev.type == "cpu" else torch.bfloat16
    grad = torch.zeros(lay.total, dtype=torch.float32, device=dev)
    w = Weights(cfg, init_flat(cfg, lay, dev, dtype=dtype, seed=seed, std=0.05), lay, grad)
    rng = np.random.default_rng(seed)
    pre = rng.integers(1, cfg.vocab_size, prefix)
    seqs = [np.r_[pre, rng.integers(1, cfg.vocab_size, int(tail * (0.5 + rng.random())))] for _ in range(n_seqs)]
    wts = [rng.normal(size=len(s)).astype(np.float32) for s in seqs]

    def score(idx, share, with_grad):
        flat = np.concatenate([seqs[i] for i in idx])
        cu = np.r_[0, np.cumsum([len(seqs[i]) for i in idx])]
        m = np.concatenate([np.r_[0.0, np.ones(len(seqs[i]) - 1)] for i in idx]).astype(np.float32)
        a = np.concatenate([wts[i] for i in idx])
        mb = build_microbatch(flat, cu, None, m, a, np.zeros(len(flat), np.float32), pad_to=8, share=share)
        d = mb.to_device(dev)
        grad.zero_()
        with torch.set_grad_enabled(with_grad):
            lp, _ = forward_tree(w, d.batch, ckpt=False)
            if with_grad:
                (lp.float() * d.adv.float() * d.w.float()).sum().backward()
        # pairs are unique (row, label): map back to flat positions through pair weights per sequence
        return lp.detach().float().cpu().numpy(), d, grad.clone() if with_grad else None

    alone = [score([i], True, False)[0] for i in range(n_seqs)]
    packed, _, g_packed = score(list(range(n_seqs)), False, True)
    tree, d_tree, g_tree = score(list(range(n_seqs)), True, True)
    a_cat = np.concatenate(alone)
    # packed scores every position; the tree scores unique (row, label) pairs: compare via sums
    # of each sequence's logprobs, which both reproduce exactly once per position
    out = {"positions": int(sum(len(s) - 1 for s in seqs)), "tree_pairs": int(len(tree)),
           "packed_vs_alone_max": float(np.abs(packed - a_cat).max()),
           "tree_total_vs_alone": float(abs(float(np.dot(d_tree.w.float().cpu().numpy(), tree)) - float(a_cat.sum()))),
           "grad_rel_l2_tree_vs_packed": float((g_tree - g_packed).norm() / g_packed.norm().clamp_min(1e-30))}
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m octopus_b200.tools.tree_check")
    ap.add_argument("--preset", default="tiny")
    ap.add_argument("--n-seqs", type=int, default=4)
    ap.add_argument("--prefix", type=int, default=300)
    ap.add_argument("--tail", type=int, default=200)
    ap.add_argument("--layers", type=int, default=0)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--cpu", action="store_true")
    args = ap.parse_args(argv)
    import torch

    dev = "cpu" if args.cpu or not torch.cuda.is_available() else "cuda"
    print(json.dumps(run(args.preset, args.n_seqs, args.prefix, args.tail, args.layers, dev, args.seed)))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
