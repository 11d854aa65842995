"""Actor for hybrid models (models.hybrid): full-parameter training of the dense part
(embedding, attention layers, head: flat buffers, as the decoder actor) and of every linear-
recurrence layer's tensors, with one AdamW step and one global gradient-norm clip over all
of them.

  weights   the dense decoder Weights (HF save / load of the dense part, checkpoints)
  hw        the HybridWeights the colocated serving.hybrid_engine.HybridEngine reads; the
            optimizer writes the compute copies in place, so the engine serves the new
            weights after each step
Micro-batches run models.hybrid.hybrid_forward over their prefix tree, or chunk-major
(rl.chunk_major: kept attention rows, recurrent states and conv rows across chunks) when a
tree has more rows than `chunk_tokens`.  Linear-layer optimizer state travels in recover
checkpoints (`extra_state`), and `save_hf` writes the linear tensors beside the dense
safetensors.

Reference parity (behaviour): training of Qwen3.5 / Qwen3-Next hybrids by the reference's
actor (`octopus/rl/actor.py`, `model_hooks.py:32-87`: GDN layers trained through the tree
recurrence; full-parameter or LoRA, full-parameter here).
"""
from __future__ import annotations

import os
import time

import torch

from .. import ops
from ..models.hybrid import HybridConfig, HybridWeights, hybrid_forward
from .actor import OptimConfig
from .chunk_major import chunk_major_forward
from .loss import PPOConfig, ppo_loss


class HybridActor:
    def __init__(self, hc: HybridConfig, device="cuda", *, optim: OptimConfig | None = None,
                 ppo: PPOConfig | None = None, seed: int = 0, dtype=torch.bfloat16, ckpt: bool = True,
                 temperature: float = 1.0):
        self.cfg = hc.base
        self.hc = hc
        self.device = torch.device(device)
        self.optim = optim or OptimConfig()
        self.ppo = ppo or PPOConfig()
        self.hw = HybridWeights(hc, self.device, dtype=dtype, seed=seed)
        self.weights = self.hw.dense
        self.layout = self.hw.layout
        self.flat16 = self.hw.dense.flat
        mdt = torch.float64 if dtype == torch.float64 else torch.float32
        self.master = self.flat16.to(mdt)
        self.grad = self.hw.grad
        self.exp_avg = torch.zeros_like(self.master)
        self.exp_avg_sq = torch.zeros_like(self.master)
        # linear-layer tensors: fp32 masters of the compute copies, and the fp32 parameters
        self.lin_master = {k: t.detach().to(mdt) for k, t in self.hw.t.items()}
        self.lin_m = {k: torch.zeros_like(v) for k, v in self.lin_master.items()}
        self.lin_v = {k: torch.zeros_like(v) for k, v in self.lin_master.items()}
        self.p_m = {k: torch.zeros_like(p) for k, p in self.hw.fp32.items()}
        self.p_v = {k: torch.zeros_like(p) for k, p in self.hw.fp32.items()}
        self.step_count = 0
        self.version = 0
        self.ckpt = ckpt
        self.temperature = temperature
        self.chunk_tokens = 0

    # ------------------------------------------------------------------ knobs
    def set_memory(self, ckpt_block: int = 1, act_gpu_bytes=None, chunk_tokens: int = 0, seq_tile: int = 0):
        """Chunk-major training bounds activation memory here; block checkpointing, host
        activations and sequence tiles are decoder-actor knobs (ignored)."""
        self.chunk_tokens = max(0, int(chunk_tokens))

    def _chunked(self, mb) -> bool:
        return bool(self.chunk_tokens) and mb.n_tree > self.chunk_tokens

    def zero_grad(self):
        self.grad.zero_()
        for t in self.hw.t.values():
            t.main_grad.zero_()
        for p in self.hw.fp32.values():
            p.grad = None

    def extra_grads(self) -> list:
        """Gradient tensors outside the flat buffer, in a fixed order (data-parallel reduce);
        absent fp32 parameter gradients are created as zeros."""
        for p in self.hw.fp32.values():
            if p.grad is None:
                p.grad = torch.zeros_like(p)
        return [t.main_grad for t in self.hw.t.values()] + [p.grad for p in self.hw.fp32.values()]

    def reload_master(self):
        self.master.copy_(self.flat16.to(self.master.dtype))
        for k, t in self.hw.t.items():
            self.lin_master[k].copy_(t.detach().to(self.lin_master[k].dtype))

    # ------------------------------------------------------------------ step
    def forward_backward(self, mbs, denom: float | None = None) -> dict:
        denom = denom if denom is not None else float(sum(mb.pair_w.sum() for mb in mbs))
        stats = {}
        for mb in mbs:
            d = mb.to_device(self.device)
            if self._chunked(mb):
                logp, ent = chunk_major_forward(self.hw, mb, self.chunk_tokens, self.temperature)
            else:
                logp, ent = hybrid_forward(self.hw, d.batch, self.temperature)
            loss, st = ppo_loss(logp, ent, d.adv, d.w, d.behav, None, denom, self.ppo)
            loss.backward()
            for k, v in st.items():
                stats[k] = stats.get(k, 0.0) + v.detach() * (1.0 if k == "tokens" else float(mb.pair_w.sum()))
            stats["loss"] = stats.get("loss", 0.0) + loss.detach()
        stats.setdefault("loss", torch.zeros((), device=self.device))
        tok = float(sum(mb.pair_w.sum() for mb in mbs)) or 1.0
        return {k: (v if k in ("tokens", "loss") else v / tok) for k, v in stats.items()}

    def optimizer_step(self) -> torch.Tensor:
        """One global norm over every gradient, then AdamW on every parameter group."""
        self.step_count += 1
        o = self.optim
        sq = torch.zeros(1, dtype=torch.float32, device=self.device)
        ops.sqnorm_(self.grad, sq)
        for t in self.hw.t.values():
            ops.sqnorm_(t.main_grad.reshape(-1), sq)
        for p in self.hw.fp32.values():
            if p.grad is not None:
                ops.sqnorm_(p.grad.reshape(-1), sq)
        kw = dict(lr=o.lr, betas=o.betas, eps=o.eps, weight_decay=o.weight_decay, step=self.step_count, sqnorm=sq,
                  max_norm=o.max_grad_norm)
        ops.adamw_(self.master, self.grad, self.exp_avg, self.exp_avg_sq, self.flat16, **kw)
        for k, t in self.hw.t.items():
            ops.adamw_(self.lin_master[k].view(-1), t.main_grad.view(-1).to(self.lin_master[k].dtype),
                       self.lin_m[k].view(-1), self.lin_v[k].view(-1), t.view(-1), **kw)
        with torch.no_grad():
            for k, p in self.hw.fp32.items():
                g = p.grad if p.grad is not None else torch.zeros_like(p)
                ops.adamw_(p.data.view(-1), g.view(-1), self.p_m[k].view(-1), self.p_v[k].view(-1), None, **kw)
        self.version += 1
        return sq

    def train_step(self, mbs) -> dict:
        t0 = time.perf_counter()
        self.zero_grad()
        stats = self.forward_backward(mbs)
        sq = self.optimizer_step()
        stats["grad_norm"] = sq.sqrt()
        stats["train_s"] = time.perf_counter() - t0
        return stats

    # ------------------------------------------------------------------ persistence
    def extra_state(self) -> dict:
        """Linear-layer parameters and optimizer state (recover checkpoints)."""
        c = lambda d: {k: v.detach().cpu().clone() for k, v in d.items()}  # noqa: E731
        return {"t": c(self.hw.t), "fp32": c(self.hw.fp32), "lin_master": c(self.lin_master), "lin_m": c(self.lin_m),
                "lin_v": c(self.lin_v), "p_m": c(self.p_m), "p_v": c(self.p_v)}

    def load_extra_state(self, st: dict):
        with torch.no_grad():
            for name, dst in (("t", self.hw.t), ("fp32", self.hw.fp32), ("lin_master", self.lin_master),
                              ("lin_m", self.lin_m), ("lin_v", self.lin_v), ("p_m", self.p_m), ("p_v", self.p_v)):
                for k, v in st[name].items():
                    dst[k].copy_(v.to(dst[k].device))

    def save_hf(self, path: str):
        """Dense part as HF safetensors, linear-layer tensors in hybrid_linear.safetensors."""
        from safetensors.torch import save_file

        from ..models.decoder import save_hf

        save_hf(self.weights, path)
        tensors = {k: v.detach().cpu().contiguous() for k, v in self.hw.t.items()}
        tensors.update({k: v.detach().cpu().contiguous() for k, v in self.hw.fp32.items()})
        save_file(tensors, os.path.join(path, "hybrid_linear.safetensors"))


class HybridLoRAActor:
    """LoRA training of a hybrid model (models.hybrid_lora): the base is frozen (no weight
    gradients, no master or optimizer state for it); AdamW runs on the adapters' flat fp32
    master; `hw` is the serving copy (base + s B A) the colocated hybrid engine reads,
    refreshed after every optimizer step."""

    def __init__(self, hc: HybridConfig, device="cuda", *, r: int = 32, alpha: float = 32.0,
                 optim: OptimConfig | None = None, ppo: PPOConfig | None = None, seed: int = 0, dtype=torch.bfloat16,
                 ckpt: bool = True, temperature: float = 1.0):
        from ..models.hybrid_lora import HybridLoRA

        self.cfg, self.hc = hc.base, hc
        self.device = torch.device(device)
        self.optim = optim or OptimConfig()
        self.ppo = ppo or PPOConfig()
        self.base = HybridWeights(hc, self.device, dtype=dtype, seed=seed, grads=False)   # frozen
        self.hw = HybridWeights(hc, self.device, dtype=dtype, seed=seed, grads=False)     # serving copy
        self.lora = HybridLoRA(hc, r, alpha, self.device, dtype, seed)
        self.weights = self.hw.dense
        self.layout = self.hw.layout
        self.master, self.grad = self.lora.master, self.lora.grad
        self.exp_avg, self.exp_avg_sq = torch.zeros_like(self.master), torch.zeros_like(self.master)
        self.step_count = 0
        self.version = 0
        self.ckpt = ckpt
        self.temperature = temperature
        self.optimizer_merge()

    def set_memory(self, ckpt_block: int = 1, act_gpu_bytes=None, chunk_tokens: int = 0, seq_tile: int = 0):
        if chunk_tokens:
            raise ValueError("chunk-major training of hybrid LoRA adapters is not supported")

    def zero_grad(self):
        self.grad.zero_()

    def reload_master(self):
        """After loading base weights (HF) into `base`: adapters keep their master."""
        self.optimizer_merge()

    def optimizer_merge(self):
        """hw <- base with s B A added to every adapted tensor."""
        with torch.no_grad():
            self.hw.dense.flat.copy_(self.base.dense.flat)
            for k, t in self.base.t.items():
                self.hw.t[k].copy_(t)
            for k, p in self.base.fp32.items():
                self.hw.fp32[k].copy_(p)
            self.lora.merge_into(self.base, self.hw)

    def forward_backward(self, mbs, denom: float | None = None) -> dict:
        denom = denom if denom is not None else float(sum(mb.pair_w.sum() for mb in mbs))
        stats = {}
        for mb in mbs:
            d = mb.to_device(self.device)
            logp, ent = hybrid_forward(self.base, d.batch, self.temperature, lora=self.lora)
            loss, st = ppo_loss(logp, ent, d.adv, d.w, d.behav, None, denom, self.ppo)
            loss.backward()
            for k, v in st.items():
                stats[k] = stats.get(k, 0.0) + v.detach() * (1.0 if k == "tokens" else float(mb.pair_w.sum()))
            stats["loss"] = stats.get("loss", 0.0) + loss.detach()
        stats.setdefault("loss", torch.zeros((), device=self.device))
        tok = float(sum(mb.pair_w.sum() for mb in mbs)) or 1.0
        return {k: (v if k in ("tokens", "loss") else v / tok) for k, v in stats.items()}

    def optimizer_step(self) -> torch.Tensor:
        self.step_count += 1
        o = self.optim
        sq = torch.zeros(1, dtype=torch.float32, device=self.device)
        ops.sqnorm_(self.grad, sq)
        ops.adamw_(self.master, self.grad, self.exp_avg, self.exp_avg_sq, self.lora.flat16, lr=o.lr, betas=o.betas,
                   eps=o.eps, weight_decay=o.weight_decay, step=self.step_count, sqnorm=sq, max_norm=o.max_grad_norm)
        self.optimizer_merge()
        self.version += 1
        return sq

    def train_step(self, mbs) -> dict:
        t0 = time.perf_counter()
        self.zero_grad()
        stats = self.forward_backward(mbs)
        sq = self.optimizer_step()
        stats["grad_norm"] = sq.sqrt()
        stats["train_s"] = time.perf_counter() - t0
        return stats

    def extra_state(self) -> dict:
        return {}

    def load_extra_state(self, st: dict):
        """After a recover load (adapter master restored): compute copy and serving weights."""
        self.lora.refresh_compute()
        self.optimizer_merge()

    def save_hf(self, path: str):
        """The merged serving weights (dense HF safetensors + hybrid_linear.safetensors)."""
        from safetensors.torch import save_file

        from ..models.decoder import save_hf

        save_hf(self.weights, path)
        tensors = {k: v.detach().cpu().contiguous() for k, v in self.hw.t.items()}
        tensors.update({k: v.detach().cpu().contiguous() for k, v in self.hw.fp32.items()})
        save_file(tensors, os.path.join(path, "hybrid_linear.safetensors"))


__all__ = ["HybridActor", "HybridLoRAActor"]
