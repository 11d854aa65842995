"""Recover checkpoints: HF-layout safetensors weights + sharded optimizer state + step,
RNG and dataloader position; atomic directory swap; spool commit after each write.

Layout of ``<dir>/recover/``:
  weights/            HF safetensors (model-0000x-of-0000y.safetensors + index + config.json)
  optim-rank<r>.pt    this rank's fp32 master / exp_avg / exp_avg_sq shards + layout hash
  state.json          {step, version, world, rng (python, numpy, torch cpu), dataloader}

A checkpoint is written to ``recover.tmp`` and renamed over ``recover`` only when every
rank has finished (rank 0 renames after a barrier), so a crash mid-write leaves the
previous checkpoint intact.  ``load`` restores weights into the flat buffers, the
optimizer shards (the world size must match) and the RNG state.

Reference parity (behaviour): AReaL recover checkpoints configured by
`octopus/rl/grpo.yaml:162-169` (LoRA + optimizer + dataloader every step) and
`octopus/rl/train.py:78-83` (spool commit after the recover checkpoint).
"""
from __future__ import annotations

import hashlib
import json
import os
import random
import shutil

import numpy as np
import torch

from ..models.decoder import load_hf, save_hf


def _layout_hash(actor) -> str:
    h = hashlib.sha1()
    for s in actor.layout.specs:
        h.update(f"{s.name}{s.shape}{actor.layout.offsets[s.name]}".encode())
    h.update(str(actor.layout.total).encode())
    return h.hexdigest()[:16]


def _dist():
    import torch.distributed as dist

    return dist if dist.is_available() and dist.is_initialized() else None


def save(actor, root: str, step: int, dataloader_state: dict | None = None, spool=None, group=None) -> str:
    """Write a recover checkpoint; `group`: the process group that holds the actor (default:
    every rank), whose first rank writes the weights and the state."""
    dist = _dist()
    rank = dist.get_rank(group) if dist else 0
    world = dist.get_world_size(group) if dist else 1
    tmp = os.path.join(root, "recover.tmp")
    final = os.path.join(root, "recover")
    if rank == 0:
        shutil.rmtree(tmp, ignore_errors=True)
        os.makedirs(tmp, exist_ok=True)
        save_hf(actor.weights, os.path.join(tmp, "weights"))
    if dist:
        dist.barrier(group)
    opt = {"master": actor.master.cpu(), "exp_avg": actor.exp_avg.cpu(), "exp_avg_sq": actor.exp_avg_sq.cpu(),
           "step_count": actor.step_count, "layout": _layout_hash(actor)}
    if hasattr(actor, "extra_state"):  # parameters and optimizer state outside the flat layout (hybrid layers)
        opt["extra"] = actor.extra_state()
    torch.save(opt, os.path.join(tmp, f"optim-rank{rank}.pt"))
    if dist:
        dist.barrier(group)
    if rank == 0:
        state = {"step": step, "version": actor.version, "world": world,
                 "rng": {"python": repr(random.getstate()), "numpy": np.random.get_state()[1].tolist()[:8],
                         "torch": torch.get_rng_state().tolist()[:16]},
                 "dataloader": dataloader_state or {}}
        with open(os.path.join(tmp, "state.json"), "w") as f:
            json.dump(state, f)
        old = final + ".old"
        shutil.rmtree(old, ignore_errors=True)
        if os.path.exists(final):
            os.replace(final, old)
        os.replace(tmp, final)
        shutil.rmtree(old, ignore_errors=True)
        if spool is not None:
            spool.commit()
    if dist:
        dist.barrier(group)
    return final


def load(actor, root: str, group=None) -> dict:
    dist = _dist()
    rank = dist.get_rank(group) if dist else 0
    world = dist.get_world_size(group) if dist else 1
    d = os.path.join(root, "recover")
    with open(os.path.join(d, "state.json")) as f:
        state = json.load(f)
    if state["world"] != world:
        raise ValueError(f"checkpoint written by {state['world']} ranks, resuming with {world}")
    load_hf(actor.weights, os.path.join(d, "weights"))
    opt = torch.load(os.path.join(d, f"optim-rank{rank}.pt"), weights_only=False)
    if opt["layout"] != _layout_hash(actor):
        raise ValueError("checkpoint parameter layout does not match the model")
    actor.master.copy_(opt["master"].to(actor.master.device))
    actor.exp_avg.copy_(opt["exp_avg"].to(actor.exp_avg.device))
    actor.exp_avg_sq.copy_(opt["exp_avg_sq"].to(actor.exp_avg_sq.device))
    if hasattr(actor, "load_extra_state"):
        actor.load_extra_state(opt["extra"])
    actor.step_count = int(opt["step_count"])
    actor.version = int(state["version"])
    if hasattr(actor, "after_load"):  # derived buffers (e.g. full-shard bf16 weight shards)
        actor.after_load()
    return state


def exists(root: str) -> bool:
    return os.path.exists(os.path.join(root, "recover", "state.json"))
