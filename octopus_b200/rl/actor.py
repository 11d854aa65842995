"""Prefix-tree policy actor: micro-batch building, forward/backward, fused AdamW.

`build_microbatch` turns flat sequences (with mounts, loss masks, per-token advantages
and behaviour logprobs) into a prefix-tree micro-batch: tree tokens and K2 positions,
the gathered-key attention plan, and per-pair (advantage, loss weight, behaviour
logprob) obtained by summing the flat tokens that map to each (row, label) pair.

`Actor` owns the flat parameter / gradient / optimizer buffers of one model replica
and runs a training step over a list of micro-batches: one forward+backward per
micro-batch (gradients accumulate in fp32 straight from the wgrad GEMM epilogues),
then a device-side grad-norm and one fused AdamW kernel over the flat buffers that
also writes the bf16 compute copy (which the colocated rollout engine reads).

Reference parity: `octopus/rl/actor.py:41-351` (ChunkedHeadFSDPPPOActor: prefix-aware
allocation, scored positions from the rolled loss mask, once-per-call sync,
optimizer step), `octopus/rl/prefix_tree.py:424-446` (tree_inputs).
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field

import numpy as np
import torch

from .. import ops
from ..models.config import ModelConfig
from ..models.decoder import FlatLayout, TreeBatch, Weights, forward_tree, init_flat
from .chunk_major import chunk_major_forward
from ..utils.iostats import h2d
from .loss import PPOConfig, ppo_loss
from .prefix_tree import attention_plan, build_tree


@dataclass
class MicroBatch:
    """Host-side prefix-tree micro-batch."""

    tokens: np.ndarray      # [Tp] int64 (padded)
    positions: np.ndarray   # [Tp] int32
    cu_q: np.ndarray
    cu_k: np.ndarray
    key_idx: np.ndarray
    pair_row: np.ndarray
    pair_label: np.ndarray
    pair_adv: np.ndarray
    pair_w: np.ndarray
    pair_behav: np.ndarray
    n_tree: int
    n_flat: int
    plan_own: tuple | None = None  # (cu_q, cu_k, key_idx) without mounted keys (layer subsets)
    nodes: np.ndarray | None = None  # [n_nodes, 4] (start, end, parent, depth) tree nodes (recurrent layers)
    path_tail: np.ndarray | None = None  # [n_nodes, 8] last tree rows before each node on its path (-1 pad)

    def to_device(self, device) -> "DeviceMicroBatch":
        d = torch.device(device)
        T = lambda a, dt: h2d(np.ascontiguousarray(a), d, dt)  # noqa: E731
        batch = TreeBatch(T(self.tokens, torch.int64), T(self.positions, torch.int32),
                          ops.AttnPlan.build(self.cu_q, self.cu_k, self.key_idx, d),
                          T(self.pair_row, torch.int64), T(self.pair_label, torch.int64))
        batch.nodes, batch.path_tail = self.nodes, self.path_tail
        return DeviceMicroBatch(batch, T(self.pair_adv, torch.float32), T(self.pair_w, torch.float32),
                                T(self.pair_behav, torch.float32))


@dataclass
class DeviceMicroBatch:
    batch: TreeBatch
    adv: torch.Tensor
    w: torch.Tensor
    behav: torch.Tensor


def build_microbatch(flat: np.ndarray, cu, mounts: dict | None, loss_mask: np.ndarray, adv: np.ndarray,
                     behav_logp: np.ndarray, pad_to: int = 128, share: bool = True) -> MicroBatch:
    """loss_mask/adv/behav_logp are per flat token (token p is trained when mask[p])."""
    flat = np.asarray(flat, dtype=np.int64)
    n = len(flat)
    scored = np.zeros(n, dtype=bool)
    scored[:-1] = loss_mask[1:].astype(bool)
    tree = build_tree(flat, cu, mounts, scored, share=share)
    plan = attention_plan(tree, True, pad_to)
    Tp = plan.padded_tokens
    toks = np.zeros(Tp, np.int64)
    toks[: tree.num_tokens] = tree.tokens
    pos = np.zeros(Tp, np.int32)
    pos[: tree.num_tokens] = tree.positions
    P = len(tree.pair_row)
    sel = np.flatnonzero(tree.flat_pair >= 0)
    pid = tree.flat_pair[sel]
    nxt = sel + 1  # the trained token of flat position p is p + 1
    w = np.bincount(pid, minlength=P).astype(np.float32)
    a = np.bincount(pid, weights=adv[nxt], minlength=P).astype(np.float32)
    b = np.bincount(pid, weights=behav_logp[nxt], minlength=P).astype(np.float32)
    nz = np.maximum(w, 1.0)
    # tree nodes for recurrent layers (+ one node covering the padding rows)
    nodes = [(nd.start, nd.end, nd.parent, nd.depth) for nd in tree.nodes]
    if Tp > tree.num_tokens:
        nodes.append((tree.num_tokens, Tp, -1, 0))
    tails = np.full((len(nodes), 8), -1, np.int64)
    for k, nd in enumerate(tree.nodes):
        if nd.parent >= 0:
            pr = tree.path_rows(nd.parent)[-8:]
            tails[k, 8 - len(pr):] = pr
    return MicroBatch(toks, pos, plan.cu_q, plan.cu_k, plan.key_idx, tree.pair_row.astype(np.int64),
                      tree.pair_label.astype(np.int64), a / nz, w, b / nz, tree.num_tokens, n,
                      nodes=np.asarray(nodes, np.int64).reshape(-1, 4), path_tail=tails)


@dataclass
class OptimConfig:
    lr: float = 2e-5
    betas: tuple = (0.9, 0.999)
    eps: float = 1e-8
    weight_decay: float = 0.0
    max_grad_norm: float = 1.0


class Actor:
    """Single-replica actor over flat buffers (the FSDP actor shards the same layout)."""

    def __init__(self, cfg: ModelConfig, device="cuda", *, optim: OptimConfig | None = None,
                 ppo: PPOConfig | None = None, seed: int = 0, dtype=torch.bfloat16, ckpt: bool = True,
                 temperature: float = 1.0):
        self.cfg = cfg
        self.device = torch.device(device)
        self.optim = optim or OptimConfig()
        self.ppo = ppo or PPOConfig()
        self.layout = FlatLayout(cfg)
        self.flat16 = init_flat(cfg, self.layout, self.device, dtype=dtype, seed=seed)
        self.master = self.flat16.float() if dtype != torch.float64 else self.flat16.clone()
        self.grad = torch.zeros(self.layout.total, dtype=torch.float32 if dtype != torch.float64 else dtype,
                                device=self.device)
        self.exp_avg = torch.zeros_like(self.master)
        self.exp_avg_sq = torch.zeros_like(self.master)
        self.weights = Weights(cfg, self.flat16, self.layout, self.grad)
        self.step_count = 0
        self.ckpt = ckpt
        self.temperature = temperature
        self.version = 0
        self.ckpt_block = 1          # block checkpoint: keep every k-th layer input
        self.chunk_tokens = 0        # chunk-major training of micro-batches larger than this (0: off)
        self.host_acts = None        # HostActivations: saved activations past a GPU budget in pinned host memory

    def set_memory(self, ckpt_block: int = 1, act_gpu_bytes: int | None = None, chunk_tokens: int = 0,
                   seq_tile: int = 0):
        """Trainer memory knobs: block checkpointing, host-resident saved activations and
        chunk-major training (micro-batches of more than chunk_tokens tree rows run through
        the model chunk by chunk: rl.chunk_major) and sequence tiles (each layer's
        o-projection and MLP in checkpointed tiles of seq_tile rows)."""
        from ..utils.pinned_slab import HostActivations, check_checkpointing

        self.ckpt_block = max(1, int(ckpt_block))
        self.chunk_tokens = max(0, int(chunk_tokens))
        self.seq_tile = max(0, int(seq_tile))  # o-projection + MLP in checkpointed row tiles (0: off)
        self.host_acts = HostActivations(act_gpu_bytes) if act_gpu_bytes is not None else None
        check_checkpointing(self.ckpt, self.host_acts)

    def zero_grad(self):
        self.grad.zero_()

    def reload_master(self):
        """fp32 master <- compute weights (after loading a checkpoint into the compute buffer)."""
        off = getattr(self, "off", 0)
        self.master.copy_(self.flat16[off: off + self.master.numel()].to(self.master.dtype))

    def forward_backward(self, mbs: list[MicroBatch], denom: float | None = None) -> dict:
        denom = denom if denom is not None else float(sum(mb.pair_w.sum() for mb in mbs))
        stats = {}
        import contextlib

        for mb in mbs:
            d = mb.to_device(self.device)
            host = getattr(self, "host_acts", None)
            with host if host is not None else contextlib.nullcontext():
                if self._chunked(mb):
                    logp, ent = chunk_major_forward(self.weights, mb, self.chunk_tokens, self.temperature)
                else:
                    logp, ent = forward_tree(self.weights, d.batch, self.temperature, ckpt=self.ckpt,
                                             ckpt_block=getattr(self, "ckpt_block", 1),
                                             seq_tile=getattr(self, "seq_tile", 0))
                loss, st = ppo_loss(logp, ent, d.adv, d.w, d.behav, None, denom, self.ppo)
            loss.backward()
            for k, v in st.items():
                stats[k] = stats.get(k, 0.0) + v.detach() * (1.0 if k == "tokens" else float(mb.pair_w.sum()))
            stats["loss"] = stats.get("loss", 0.0) + loss.detach()
        stats.setdefault("loss", torch.zeros((), device=self.device))  # a rank with no micro-batch this step
        tok = float(sum(mb.pair_w.sum() for mb in mbs)) or 1.0
        return {k: (v if k in ("tokens", "loss") else v / tok) for k, v in stats.items()}

    def _chunked(self, mb) -> bool:
        ct = getattr(self, "chunk_tokens", 0)
        return bool(ct) and self.ckpt and mb.n_tree > ct

    def optimizer_step(self) -> torch.Tensor:
        """Grad-norm clip + AdamW; returns the (device) squared grad norm."""
        self.step_count += 1
        sq = torch.zeros(1, dtype=torch.float32, device=self.device)
        ops.sqnorm_(self.grad, sq)
        o = self.optim
        ops.adamw_(self.master, self.grad, self.exp_avg, self.exp_avg_sq, self.flat16, lr=o.lr, betas=o.betas,
                   eps=o.eps, weight_decay=o.weight_decay, step=self.step_count, sqnorm=sq,
                   max_norm=o.max_grad_norm)
        self.version += 1
        return sq

    def train_step(self, mbs: list[MicroBatch]) -> dict:
        t0 = time.perf_counter()
        self.zero_grad()
        stats = self.forward_backward(mbs)
        sq = self.optimizer_step()
        stats["grad_norm"] = sq.sqrt()
        stats["train_s"] = time.perf_counter() - t0
        return stats


class LoRAActor(Actor):
    """Actor that trains low-rank adapters on a frozen base (octopus_b200.models.lora).

    The base bf16 weights get no gradient (no weight-gradient GEMMs, no fp32 master or
    optimizer state for them); AdamW runs on the adapters' flat fp32 master.  `serving`
    holds W + s B A for the rollout engine, refreshed after every optimizer step (the
    trainer -> rollout weight sync)."""

    def __init__(self, cfg: ModelConfig, device="cuda", *, lora=None, optim: OptimConfig | None = None,
                 ppo: PPOConfig | None = None, seed: int = 0, dtype=torch.bfloat16, ckpt: bool = True,
                 temperature: float = 1.0):
        from ..models.lora import LoRA, merge

        self.cfg = cfg
        self.device = torch.device(device)
        self.optim = optim or OptimConfig()
        self.ppo = ppo or PPOConfig()
        self.layout = FlatLayout(cfg)
        self.base16 = init_flat(cfg, self.layout, self.device, dtype=dtype, seed=seed)
        self.base = Weights(cfg, self.base16, self.layout)          # frozen: no main_grad
        self.lora = LoRA(cfg, lora, self.device, dtype, seed)
        self.master, self.grad = self.lora.master, self.lora.grad
        self.exp_avg, self.exp_avg_sq = self.lora.exp_avg, self.lora.exp_avg_sq
        self.flat16 = self.lora.flat16
        self.serving = Weights(cfg, self.base16.clone(), self.layout)
        self._merge = merge
        self._merge(self.base, self.lora, self.serving)
        self.weights = self.serving   # what the colocated engine reads
        self.step_count = 0
        self.ckpt = ckpt
        self.temperature = temperature
        self.version = 0
        self.ckpt_block = 1
        self.chunk_tokens = 0
        self.host_acts = None

    def forward_backward(self, mbs: list[MicroBatch], denom: float | None = None) -> dict:
        denom = denom if denom is not None else float(sum(mb.pair_w.sum() for mb in mbs))
        stats = {}
        for mb in mbs:
            d = mb.to_device(self.device)
            if self._chunked(mb):
                logp, ent = chunk_major_forward(self.base, mb, self.chunk_tokens, self.temperature, lora=self.lora)
            else:
                logp, ent = forward_tree(self.base, d.batch, self.temperature, ckpt=self.ckpt,
                                         ckpt_block=self.ckpt_block, lora=self.lora,
                                         seq_tile=getattr(self, "seq_tile", 0))
            loss, st = ppo_loss(logp, ent, d.adv, d.w, d.behav, None, denom, self.ppo)
            loss.backward()
            for k, v in st.items():
                stats[k] = stats.get(k, 0.0) + v.detach() * (1.0 if k == "tokens" else float(mb.pair_w.sum()))
            stats["loss"] = stats.get("loss", 0.0) + loss.detach()
        stats.setdefault("loss", torch.zeros((), device=self.device))
        tok = float(sum(mb.pair_w.sum() for mb in mbs)) or 1.0
        return {k: (v if k in ("tokens", "loss") else v / tok) for k, v in stats.items()}

    def optimizer_step(self) -> torch.Tensor:
        sq = super().optimizer_step()   # AdamW on the adapters' master -> lora.flat16
        self.optimizer_merge()
        return sq

    def optimizer_merge(self):
        """serving <- base + s B A (after an update or a base reload)."""
        self.serving.flat.copy_(self.base16)
        self._merge(self.base, self.lora, self.serving)

    def reload_master(self):
        self.lora.master.copy_(self.lora.flat16.to(self.lora.master.dtype))
