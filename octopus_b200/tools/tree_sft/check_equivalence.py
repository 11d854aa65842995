"""Check: the tree loss (root computed once) equals the sum of the flat losses over
root + child sequences, in value and in adapter gradients.

    python -m octopus_b200.tools.tree_sft.check_equivalence [--preset qwen2.5-7b --layers 2] [--root 300]
        [--child 120] [--fp32]

Random tokens: a root of --root tokens whose second half is labelled (pre-fork turns,
trained once: in the tree's root, in the first flat row), three children of --child tokens
whose last two thirds are labelled.  Adapters get non-zero B so every matrix has a gradient.
Prints the relative differences (fp32 separates rounding from real mismatches).

Reference parity (behaviour): `octopus/tools/tree_sft/check_equivalence.py:1-67`.
"""
from __future__ import annotations

import argparse
import json

import numpy as np
import torch

from .encode import IGNORE
from .train import _microbatch, labelled_ce


def synthetic_tree(vocab: int, root: int = 300, child: int = 120, n_children: int = 3, seed: int = 0) -> dict:
    rng = np.random.default_rng(seed)
    root_ids = rng.integers(1, vocab, root).tolist()
    root_labels = [IGNORE] * (root // 2) + root_ids[root // 2:]
    children = []
    for _ in range(n_children):
        ids = rng.integers(1, vocab, child).tolist()
        children.append({"kind": "branch", "ids": ids, "labels": [IGNORE] * (child // 3) + ids[child // 3:]})
    children[0]["kind"] = "join"
    return {"root_ids": root_ids, "root_labels": root_labels, "children": children}


def compare(actor, enc: dict) -> dict:
    """Loss and adapter-gradient differences of tree vs flat on one encoded tree."""
    from .encode import flat_rows

    actor.zero_grad()
    t_loss, t_n = labelled_ce(actor, _microbatch([(r["input_ids"], r["labels"]) for r in flat_rows(enc)]))
    t_loss.backward()
    tg = actor.grad.detach().double().clone()
    actor.zero_grad()
    f_loss, f_n = 0.0, 0
    for r in flat_rows(enc):
        loss, n = labelled_ce(actor, _microbatch([(r["input_ids"], r["labels"])], share=False))
        loss.backward()
        f_loss, f_n = f_loss + float(loss.detach()), f_n + n
    fg = actor.grad.detach().double().clone()
    actor.zero_grad()
    return {"tokens_tree": t_n, "tokens_flat": f_n, "loss_tree": float(t_loss.detach()), "loss_flat": f_loss,
            "loss_rel_diff": abs(float(t_loss.detach()) - f_loss) / max(abs(f_loss), 1e-30),
            "grad_rel_diff": float((tg - fg).norm() / fg.norm().clamp_min(1e-30)), "grad_norm": float(fg.norm())}


def make_actor(cfg, device, dtype, r: int = 8, seed: int = 0):
    from ...models.lora import LoRAConfig
    from ...rl.actor import LoRAActor

    actor = LoRAActor(cfg, device, lora=LoRAConfig(r=r, alpha=2.0 * r), dtype=dtype, seed=seed)
    g = torch.Generator(device="cpu").manual_seed(seed + 1)
    with torch.no_grad():
        for name, t in actor.lora.t.items():
            if name.endswith(".B"):  # non-zero B: every adapter matrix gets a gradient
                t.copy_((torch.randn(t.shape, generator=g) * 1e-3).to(t.dtype))
    actor.reload_master()
    return actor


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m octopus_b200.tools.tree_sft.check_equivalence")
    ap.add_argument("--preset", default="qwen2.5-7b")
    ap.add_argument("--layers", type=int, default=2)
    ap.add_argument("--root", type=int, default=300)
    ap.add_argument("--child", type=int, default=120)
    ap.add_argument("--fp32", action="store_true")
    args = ap.parse_args(argv)
    from ...models.config import get_config

    cuda = torch.cuda.is_available()
    cfg = get_config(args.preset, layers=args.layers)
    actor = make_actor(cfg, "cuda" if cuda else "cpu", torch.float32 if args.fp32 or not cuda else torch.bfloat16)
    print(json.dumps(compare(actor, synthetic_tree(cfg.vocab_size, args.root, args.child))))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
