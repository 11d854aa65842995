"""LoRA SFT on encoded fork trees: method "tree" or "flat".

    python -m octopus_b200.tools.tree_sft.train --data encoded.jsonl --out DIR [--method tree|flat]
        [--model HF_DIR | --preset tiny] [--rank 16] [--alpha 32] [--lr 1e-4] [--epochs 2]
        [--per-step 8] [--warmup 0.05] [--seed 0] [--max-trees 0] [--chunk-tokens 0]

tree  each tree is one prefix-tree micro-batch (rl.actor.build_microbatch over root + each
      child): the root's rows exist once and every child attends to them through the tree
      attention plan; the tree's loss is its mean CE over its labelled tokens (one tree =
      one unit of weight), averaged over the `--per-step` trees of a step
flat  one micro-batch per child (root + child, the root's labels in the join row only);
      the step's loss is the summed CE over its `--per-step` samples divided by their
      labelled tokens
Both train the same adapters (all linear projections) with AdamW, a cosine schedule with
linear warm-up and a gradient-norm clip of 1.0.  Under torchrun each step's trees (or
samples) are split over the ranks and the adapters' flat gradient buffer is summed with
one all-reduce, so K GPUs give the single-GPU update.  A tree too large for the device is
skipped (with this rank's partial gradients of the step) and logged.  Adapters are saved
in PEFT layout after every epoch and at the end.

Reference parity (behaviour): `octopus/tools/tree_sft/train_tree.py:1-123` (tree method,
per-tree mean, OOM skip, rank split with summed gradients) and `train_flat.py:1-128` (flat
method with the same labelled CE, normalised over the accumulated batch).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import random
import time
from pathlib import Path

import numpy as np
import torch

from .encode import IGNORE, flat_rows


def _microbatch(seqs: list[tuple[list[int], list[int]]], share: bool = True):
    from ...rl.actor import build_microbatch

    flat = np.concatenate([np.asarray(ids, np.int64) for ids, _ in seqs])
    labels = np.concatenate([np.asarray(lab, np.int64) for _, lab in seqs])
    cu = np.cumsum([0] + [len(ids) for ids, _ in seqs])
    mask = (labels != IGNORE).astype(np.float32)
    mask[cu[:-1]] = 0.0  # a sequence's first token has no prediction
    n = len(flat)
    return build_microbatch(flat, cu, None, mask, np.ones(n, np.float32), np.zeros(n, np.float32), share=share)


def tree_microbatch(enc: dict):
    """One prefix-tree micro-batch of a tree (root shared by all children)."""
    return _microbatch([(r["input_ids"], r["labels"]) for r in flat_rows(enc)], share=True)


def flat_microbatches(enc: dict) -> list:
    """One micro-batch per flat row."""
    return [_microbatch([(r["input_ids"], r["labels"])], share=False) for r in flat_rows(enc)]


def labelled_ce(actor, mb) -> tuple[torch.Tensor, int]:
    """(summed CE over the micro-batch's labelled tokens, their count) with the actor's
    weights (and adapters)."""
    from ...models.decoder import forward_tree
    from ...rl.chunk_major import chunk_major_forward

    lora = getattr(actor, "lora", None)
    w = actor.base if lora is not None else actor.weights
    if actor._chunked(mb):
        logp, _ = chunk_major_forward(w, mb, actor.chunk_tokens, 1.0, lora=lora)
        wt = torch.as_tensor(mb.pair_w, device=logp.device, dtype=torch.float32)
    else:
        d = mb.to_device(actor.device)
        logp, _ = forward_tree(w, d.batch, 1.0, ckpt=actor.ckpt, ckpt_block=actor.ckpt_block, lora=lora,
                               seq_tile=getattr(actor, "seq_tile", 0))
        wt = d.w
    lp = logp if logp.dtype == torch.float64 else logp.float()
    return -(lp * wt).sum(), int(round(float(mb.pair_w.sum())))


def cosine_lr(step: int, total: int, warmup: int, peak: float) -> float:
    if warmup and step < warmup:
        return peak * (step + 1) / warmup
    frac = (step - warmup) / max(1, total - warmup)
    return peak * 0.5 * (1.0 + math.cos(math.pi * min(1.0, frac)))


def _oom(e) -> bool:
    return isinstance(e, torch.cuda.OutOfMemoryError) or "out of memory" in str(e)


def train(actor, trees: list[dict], out_dir, *, method: str = "tree", epochs: int = 2, per_step: int = 8,
          lr: float = 1e-4, warmup: float = 0.05, seed: int = 0, rank: int = 0, world: int = 1, group=None,
          log=print) -> list[dict]:
    """Train actor's adapters on encoded trees; returns the per-step records."""
    import torch.distributed as dist

    rng = random.Random(seed)  # the same order on every rank
    units = trees if method == "tree" else [(t, i) for t in trees for i in range(len(t["children"]))]
    steps = epochs * math.ceil(len(units) / per_step)
    warm = int(steps * warmup)
    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    flog = (out / "train_log.jsonl").open("a") if rank == 0 else None
    recs, step, t0 = [], 0, time.time()
    for epoch in range(epochs):
        order = list(range(len(units)))
        rng.shuffle(order)
        for s0 in range(0, len(order), per_step):
            window = order[s0:s0 + per_step]
            actor.zero_grad()
            acc = torch.zeros(2, dtype=torch.float64, device=actor.device)  # loss sum, labelled tokens
            if method == "flat":  # the step's denominator: every sample's labelled tokens (all ranks)
                denom = 0
                for k in window:
                    t, i = units[k]
                    denom += sum(x != IGNORE for x in flat_rows(t)[i]["labels"][1:])
                denom = max(denom, 1)
            for k in window[rank::world]:
                try:
                    if method == "tree":
                        loss, n = labelled_ce(actor, tree_microbatch(units[k]))
                        (loss / max(n, 1) / per_step).backward()
                    else:
                        t, i = units[k]
                        loss, n = labelled_ce(actor, flat_microbatches(t)[i])
                        (loss / denom).backward()
                except (torch.cuda.OutOfMemoryError, RuntimeError) as e:
                    if not _oom(e):
                        raise
                    log(json.dumps({"skipped_oom": k, "step": step, "rank": rank}))
                    actor.zero_grad()
                    acc.zero_()
                    if torch.cuda.is_available():
                        torch.cuda.empty_cache()
                    continue
                acc += torch.tensor([float(loss.detach()), n], dtype=torch.float64, device=actor.device)
            if world > 1:  # every rank joins every step's reduce, with or without trees
                dist.all_reduce(actor.grad, group=group)
                dist.all_reduce(acc, group=group)
            actor.optim.lr = cosine_lr(step, steps, warm, lr)
            sq = actor.optimizer_step()
            step += 1
            rec = {"step": step, "epoch": epoch, "loss": float(acc[0]) / max(float(acc[1]), 1.0),
                   "tokens": int(acc[1]), "grad_norm": round(float(sq.sqrt()), 4), "lr": actor.optim.lr,
                   "elapsed_s": round(time.time() - t0, 1)}
            recs.append(rec)
            if flog is not None:
                flog.write(json.dumps(rec) + "\n")
                flog.flush()
                log(json.dumps(rec))
        if rank == 0:
            actor.lora.save_peft(str(out / f"epoch{epoch + 1}"))
    if rank == 0:
        actor.lora.save_peft(str(out / "final"))
    if flog is not None:
        flog.close()
    return recs


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m octopus_b200.tools.tree_sft.train")
    ap.add_argument("--data", required=True)
    ap.add_argument("--out", required=True)
    ap.add_argument("--method", choices=("tree", "flat"), default="tree")
    ap.add_argument("--model", default="", help="HF checkpoint directory of --preset's architecture (the base)")
    ap.add_argument("--preset", default="qwen2.5-7b")
    ap.add_argument("--rank", type=int, default=16)
    ap.add_argument("--alpha", type=float, default=32.0)
    ap.add_argument("--lr", type=float, default=1e-4)
    ap.add_argument("--epochs", type=int, default=2)
    ap.add_argument("--per-step", type=int, default=8, help="trees (tree) or samples (flat) per optimizer step")
    ap.add_argument("--warmup", type=float, default=0.05)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--max-trees", type=int, default=0)
    ap.add_argument("--chunk-tokens", type=int, default=0, help="chunk-major training of trees above this size")
    args = ap.parse_args(argv)

    import torch.distributed as dist

    from ...models.config import get_config
    from ...models.decoder import load_hf
    from ...models.lora import LoRAConfig
    from ...rl.actor import LoRAActor, OptimConfig

    world, rank = int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0"))
    cuda = torch.cuda.is_available()
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0"))) if cuda else torch.device("cpu")
    if cuda:
        torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl" if cuda else "gloo")
    trees = [json.loads(x) for x in open(args.data) if x.strip()][: args.max_trees or None]
    cfg = get_config(args.preset)  # the architecture of --model
    actor = LoRAActor(cfg, dev, lora=LoRAConfig(r=args.rank, alpha=args.alpha),
                      optim=OptimConfig(lr=args.lr, max_grad_norm=1.0),
                      dtype=torch.bfloat16 if cuda else torch.float32, seed=args.seed)
    if args.model:
        load_hf(actor.base, args.model)
        actor.optimizer_merge()
    actor.set_memory(chunk_tokens=args.chunk_tokens)
    train(actor, trees, args.out, method=args.method, epochs=args.epochs, per_step=args.per_step, lr=args.lr,
          warmup=args.warmup, seed=args.seed, rank=rank, world=world)
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
