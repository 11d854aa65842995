"""LoRA adapters for hybrid models: the attention layers' projections (qkv, o, gate/up, down,
as models.lora) and the linear-recurrence layers' input, gate, output and MLP projections
(lin_qkv, lin_z, lin_out, gu_w, down_w).  Every adapted W [out, in] gets A [r, in] (random,
scale 1/sqrt(in)) and B [out, r] (zero: step 0 is the base model) in one flat fp32 master /
bf16 compute / fp32 gradient buffer; the layer computes W x + (alpha / r) B A x.  The
beta / gate projection (a few rows) and the conv taps and gates stay frozen.

`merge_into(base, out)` writes W + s B A for every adapted tensor into another HybridWeights
(the serving copy the hybrid engine reads).

Reference parity (behaviour): LoRA on Qwen3.5's GDN projections served by the reference's
SGLang patch (`patches/apply_sglang_lora_targets.py`: fused qkvz adapters, Mamba out_proj)
and the LoRA settings of `octopus/rl/grpo.yaml` (r 32, alpha 32).
"""
from __future__ import annotations

import math

import torch

from .. import ops
from .hybrid import HybridConfig

ATTN = ("qkv_w", "o_w", "gu_w", "down_w")
LIN = ("lin_qkv", "lin_z", "lin_out", "gu_w", "down_w")


def _shapes(hc: HybridConfig) -> dict:
    cfg, C, F, H = hc.base, hc.lin_width, hc.base.ffn, hc.base.hidden
    out = {}
    for i in range(cfg.layers):
        if hc.is_linear(i):
            dims = {"lin_qkv": (3 * C, H), "lin_z": (C, H), "lin_out": (H, C), "gu_w": (2 * F, H), "down_w": (H, F)}
        else:
            dims = {"qkv_w": (cfg.qkv_width, H), "o_w": (H, cfg.q_width), "gu_w": (2 * F, H), "down_w": (H, F)}
        for k, v in dims.items():
            out[f"layers.{i}.{k}"] = v
    return out


class HybridLoRA:
    def __init__(self, hc: HybridConfig, r: int = 32, alpha: float = 32.0, device="cuda", dtype=torch.bfloat16,
                 seed: int = 0):
        self.hc, self.r, self.alpha = hc, int(r), float(alpha)
        self.scale = self.alpha / self.r
        self.shapes = _shapes(hc)
        specs, off = [], 0
        for name, (o, n) in self.shapes.items():
            for ab, shape in (("A", (self.r, n)), ("B", (o, self.r))):
                specs.append((f"{name}.{ab}", shape, off))
                off += (math.prod(shape) + 127) // 128 * 128
        self.total = off
        gdt = torch.float64 if dtype == torch.float64 else torch.float32
        dev = torch.device(device)
        self.master = torch.zeros(off, dtype=gdt, device=dev)
        g = torch.Generator(device="cpu").manual_seed(seed + 17)
        for name, shape, o in specs:
            if name.endswith(".A"):
                n = math.prod(shape)
                self.master[o:o + n] = (torch.randn(n, generator=g) / math.sqrt(shape[1])).to(gdt).to(dev)
        self.flat16 = self.master.to(dtype)
        self.grad = torch.zeros(off, dtype=gdt, device=dev)
        self.t = {}
        for name, shape, o in specs:
            n = math.prod(shape)
            v = self.flat16[o:o + n].view(shape)
            v.main_grad = self.grad[o:o + n].view(shape)
            self.t[name] = v

    def get(self, name: str):
        """(A, B, scale) of the adapted tensor `name` ("layers.<i>.<proj>"), or None."""
        if name not in self.shapes:
            return None
        return self.t[f"{name}.A"], self.t[f"{name}.B"], self.scale

    def layer(self, i: int):
        """An attention layer's (qkv, o, gu, down) adapters (the decoder layer's lora argument)."""
        return tuple(self.get(f"layers.{i}.{p}") for p in ATTN)

    def refresh_compute(self):
        self.flat16.copy_(self.master.to(self.flat16.dtype))

    def merge_into(self, base, out):
        """out[name] = base[name] + s B A for every adapted tensor (base / out: HybridWeights)."""
        for name in self.shapes:
            i = int(name.split(".")[1])
            if self.hc.is_linear(i):
                w, dst = base.t[name], out.t[name]
            else:
                w, dst = base.dense[name], out.dense[name]
            A, B = self.t[f"{name}.A"], self.t[f"{name}.B"]
            ops.gemm(B, A, b_mn=True, alpha=self.scale, residual=w, out=dst)


__all__ = ["ATTN", "HybridLoRA", "LIN"]
