"""Low-rank adapters (LoRA) on the decoder's projections, and their merge into serving
weights.

Every targeted projection W [out, in] of every layer gets A [r, in] (random, scale
1/sqrt(in)) and B [out, r] (zero, so step 0 is the base model); the layer computes
W x + (alpha / r) B A x with the base frozen (no weight gradient is computed for it).
Adapters live in one flat fp32 master buffer (AdamW on it), one flat bf16 compute buffer
and one flat fp32 gradient buffer (`main_grad` views), like the base weights.

Fused projections carry one adapter: qkv (q, k, v share A; B covers all three output
blocks), gate/up likewise.  `TARGETS` maps PEFT module names onto them; a PEFT export
writes the per-module tensors (A repeated for the fused parts, B split).

Serving: `merge(base, lora, out)` writes W + s B A for every targeted projection into
another weight set (one fused GEMM per projection: residual = W, K = r), the rollout
engine's weights after each optimizer step.

Reference parity (behaviour): `octopus/rl/lora_targets.py:27-64` (targets SGLang can
serve), `octopus/rl/zero_adapter.py:1-33` (the v0 adapter has B = 0), the LoRA settings of
`octopus/rl/grpo.yaml` (r 32, alpha 32).
"""
from __future__ import annotations

import json
import math
import os
from dataclasses import dataclass, field

import torch

from .. import ops
from .config import ModelConfig

# our projection -> PEFT module names it covers
TARGETS = {"qkv_w": ("q_proj", "k_proj", "v_proj"), "o_w": ("o_proj",), "gu_w": ("gate_proj", "up_proj"),
           "down_w": ("down_proj",)}
PEFT_PARENT = {"q_proj": "self_attn", "k_proj": "self_attn", "v_proj": "self_attn", "o_proj": "self_attn",
               "gate_proj": "mlp", "up_proj": "mlp", "down_proj": "mlp"}


def lora_targets(modules) -> tuple[str, ...]:
    """PEFT target module names ("all-linear" or a list) -> this model's adapted projections.
    A fused projection is adapted when any of its modules is named; names this decoder
    cannot serve raise."""
    if modules in ("all-linear", "all", None):
        return tuple(TARGETS)
    names = [modules] if isinstance(modules, str) else list(modules)
    known = {m: t for t, ms in TARGETS.items() for m in ms}
    bad = [n for n in names if n not in known]
    if bad:
        raise ValueError(f"LoRA targets not servable by this decoder: {bad} (known: {sorted(known)})")
    return tuple(t for t in TARGETS if any(known[n] == t for n in names))


@dataclass
class LoRAConfig:
    r: int = 32
    alpha: float = 32.0
    targets: tuple = field(default_factory=lambda: tuple(TARGETS))

    @property
    def scale(self) -> float:
        return self.alpha / self.r


def _dims(cfg: ModelConfig, t: str) -> tuple[int, int]:
    H = cfg.hidden
    return {"qkv_w": (cfg.qkv_width, H), "o_w": (H, cfg.q_width), "gu_w": (2 * cfg.ffn, H),
            "down_w": (H, cfg.ffn)}[t]


class LoRA:
    def __init__(self, cfg: ModelConfig, lcfg: LoRAConfig | None = None, device="cuda", dtype=torch.bfloat16,
                 seed: int = 0):
        self.cfg, self.lcfg = cfg, lcfg or LoRAConfig()
        self.device = torch.device(device)
        r = self.lcfg.r
        self.specs = []
        off = 0
        for i in range(cfg.layers):
            for t in self.lcfg.targets:
                o, n = _dims(cfg, t)
                for ab, shape in (("A", (r, n)), ("B", (o, r))):
                    self.specs.append((f"layers.{i}.{t}.{ab}", shape, off))
                    off += (math.prod(shape) + 127) // 128 * 128
        self.total = off
        gdt = torch.float64 if dtype == torch.float64 else torch.float32
        self.master = torch.zeros(self.total, dtype=gdt, device=self.device)
        g = torch.Generator(device="cpu").manual_seed(seed + 7)
        for name, shape, o in self.specs:
            if name.endswith(".A"):
                n = math.prod(shape)
                self.master[o:o + n] = (torch.randn(n, generator=g) / math.sqrt(shape[1])).to(gdt).to(self.device)
        self.flat16 = self.master.to(dtype)
        self.grad = torch.zeros(self.total, dtype=gdt, device=self.device)
        self.t = {}
        for name, shape, o in self.specs:
            n = math.prod(shape)
            v = self.flat16[o:o + n].view(shape)
            v.main_grad = self.grad[o:o + n].view(shape)
            self.t[name] = v
        self.exp_avg = torch.zeros_like(self.master)
        self.exp_avg_sq = torch.zeros_like(self.master)

    def layer(self, i: int):
        """(qkv, o, gu, down) adapters of layer i: (A, B, scale) or None."""
        s = self.lcfg.scale
        out = []
        for t in ("qkv_w", "o_w", "gu_w", "down_w"):
            out.append((self.t[f"layers.{i}.{t}.A"], self.t[f"layers.{i}.{t}.B"], s) if t in self.lcfg.targets
                       else None)
        return tuple(out)

    def refresh_compute(self):
        self.flat16.copy_(self.master.to(self.flat16.dtype))

    # ------------------------------------------------------------------ PEFT export
    def peft_tensors(self) -> dict:
        """PEFT-layout adapter tensors (fused projections split; A repeated)."""
        cfg = self.cfg
        out = {}
        split = {"qkv_w": [cfg.q_width, cfg.kv_width, cfg.kv_width], "gu_w": [cfg.ffn, cfg.ffn]}
        for i in range(cfg.layers):
            for t in self.lcfg.targets:
                A = self.t[f"layers.{i}.{t}.A"]
                B = self.t[f"layers.{i}.{t}.B"]
                mods = TARGETS[t]
                Bs = torch.split(B, split[t]) if t in split else (B,)
                for m, b in zip(mods, Bs):
                    pre = f"base_model.model.model.layers.{i}.{PEFT_PARENT[m]}.{m}"
                    out[f"{pre}.lora_A.weight"] = A.detach().contiguous()
                    out[f"{pre}.lora_B.weight"] = b.detach().contiguous()
        return out

    def save_peft(self, path: str, base_model: str = ""):
        from safetensors.torch import save_file

        os.makedirs(path, exist_ok=True)
        save_file({k: v.cpu().clone() for k, v in self.peft_tensors().items()},
                  os.path.join(path, "adapter_model.safetensors"))
        mods = sorted({m for t in self.lcfg.targets for m in TARGETS[t]})
        with open(os.path.join(path, "adapter_config.json"), "w") as f:
            json.dump({"peft_type": "LORA", "r": self.lcfg.r, "lora_alpha": self.lcfg.alpha, "target_modules": mods,
                       "lora_dropout": 0.0, "bias": "none", "task_type": "CAUSAL_LM",
                       "base_model_name_or_path": base_model}, f, indent=1)

    def load_peft(self, path: str):
        """Load an adapter exported by save_peft (A shared within fused projections)."""
        from safetensors.torch import load_file

        d = load_file(os.path.join(path, "adapter_model.safetensors"))
        cfg = self.cfg
        for i in range(cfg.layers):
            for t in self.lcfg.targets:
                mods = TARGETS[t]
                pre = [f"base_model.model.model.layers.{i}.{PEFT_PARENT[m]}.{m}" for m in mods]
                A = d[f"{pre[0]}.lora_A.weight"]
                B = torch.cat([d[f"{p}.lora_B.weight"] for p in pre])
                self.t[f"layers.{i}.{t}.A"].copy_(A)
                self.t[f"layers.{i}.{t}.B"].copy_(B)
        for name, shape, o in self.specs:
            n = math.prod(shape)
            self.master[o:o + n].copy_(self.t[name].reshape(-1).to(self.master.dtype))


def zero_adapter(cfg: ModelConfig, path: str, lcfg: LoRAConfig | None = None, base_model: str = ""):
    """Write the v0 adapter (B = 0: the base model exactly)."""
    LoRA(cfg, lcfg, device="cpu", dtype=torch.float32).save_peft(path, base_model)


def merge(base, lora: LoRA, out) -> None:
    """out[proj] = base[proj] + s * B @ A for every adapted projection (other tensors must
    already be in `out`).  base / out: decoder Weights."""
    s = lora.lcfg.scale
    for i in range(lora.cfg.layers):
        for t in lora.lcfg.targets:
            A = lora.t[f"layers.{i}.{t}.A"]  # [r, in]
            B = lora.t[f"layers.{i}.{t}.B"]  # [out, r]
            name = f"layers.{i}.{t}"
            # C[out, in] = s * B [out, r] @ (A [r, in] read as [K=r, N=in]) + W
            ops.gemm(B, A, b_mn=True, alpha=s, residual=base[name], out=out[name])
