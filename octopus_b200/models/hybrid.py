"""Hybrid decoders: linear-recurrence layers (gated DeltaNet, or the Mamba-2 / simple-GLA
form) interleaved with full-attention layers, trained over prefix trees.

A linear layer over a prefix tree: the tree's nodes tile its rows in pre-order; every
node continues its parent, so

* the causal conv of a node starts from the last W - 1 conv inputs on its ancestor path
  (context rows gathered from the tree, zeros at the root), and
* the recurrence of a node starts from its parent node's final state: nodes are run
  level by level (depth 0, 1, ...), each level one kernel call whose initial states are
  the previous level's final states.

Mounted rows (read_thread) reach the attention layers only: a recurrent layer keeps the
reader's own state.

Layer (gated DeltaNet, Qwen3-Next / Qwen3.5 style, one key head per value head):
    h = rmsnorm(x);  qkv, z, b, a = h W_qkv, h W_z, h W_b, h W_a
    qkv = silu(conv(qkv));  q, k = l2norm(q), l2norm(k)
    beta = sigmoid(b);  g = -exp(A_log) softplus(a + dt_bias)
    o = delta_rule(q, k, v, g, beta)            (Mamba-2 / GLA form: o = gla(q, k, v, g))
    x = x + W_out (rmsnorm_per_head(o) w_o * silu(z));  then the SwiGLU MLP
`FAMILIES` maps model families to their layer kinds; stateful families outside it raise.

Reference parity (behaviour): `octopus/rl/model_hooks.py:32-87` (families),
`octopus/rl/gdn_varlen.py`, `octopus/rl/mamba2_varlen.py`, `octopus/rl/seq_tiles.py:181-207`
(one recurrence level-call at a time, conv context rows), `octopus/rl/prefix_tree.py:303-361`.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from .. import ops
from ..ops.recurrence import causal_conv, recurrence
from .config import ModelConfig
from .decoder import FlatLayout, Weights, init_flat, layer_forward

FAMILIES = {
    "qwen2": "dense",
    "llama": "dense",
    "qwen3_next": "gdn",
    "qwen3_5": "gdn",
    "qwen3_5_moe": "gdn",
    "granitemoehybrid": "gla",
}


def family_kind(model_type: str) -> str:
    if model_type not in FAMILIES:
        raise ValueError(f"model family {model_type!r} has no hooks: recurrent layers would be trained wrong")
    return FAMILIES[model_type]


@dataclass(frozen=True)
class HybridConfig:
    base: ModelConfig        # hidden, attention heads, ffn, vocab, norms
    kind: str = "gdn"        # gdn | gla
    pattern: str = "LLLA"    # per layer (repeated): L = linear recurrence, A = full attention
    lin_heads: int = 4
    lin_dim: int = 128
    conv_width: int = 4

    def is_linear(self, i: int) -> bool:
        return self.pattern[i % len(self.pattern)] == "L"

    @property
    def lin_width(self) -> int:
        return self.lin_heads * self.lin_dim

    @property
    def ba_rows(self) -> int:
        """Rows of the beta / gate projection: 2 * heads, padded with zero rows to a multiple
        of 8 (the GEMM's tile granularity; the padding rows' outputs are never read, so their
        gradients and values stay zero)."""
        return (2 * self.lin_heads + 7) // 8 * 8


def hybrid_config(preset: str, layers: int = 0) -> HybridConfig | None:
    """Hybrid presets (None for a dense preset): "tiny-hybrid" (tests) and "hybrid-7b" (the 7B
    decoder's shape with three linear layers per attention layer, as Qwen3-Next / Qwen3.5)."""
    from .config import get_config

    kw = {"layers": layers} if layers else {}
    if preset == "tiny-hybrid":
        return HybridConfig(get_config("tiny", **kw), kind="gdn", pattern="LLLA", lin_heads=4, lin_dim=64)
    if preset == "hybrid-7b":
        return HybridConfig(get_config("qwen2.5-7b", **kw), kind="gdn", pattern="LLLA", lin_heads=16, lin_dim=128)
    return None


def _lin_specs(hc: HybridConfig, i: int):
    H, C = hc.base.hidden, hc.lin_width
    return [(f"layers.{i}.ln1", (H,), "ones"), (f"layers.{i}.lin_qkv", (3 * C, H), "normal"),
            (f"layers.{i}.lin_z", (C, H), "normal"), (f"layers.{i}.lin_ba", (hc.ba_rows, H), "ba"),
            (f"layers.{i}.lin_out", (H, C), "normal"),
            (f"layers.{i}.lin_norm", (hc.lin_dim,), "ones"), (f"layers.{i}.ln2", (H,), "ones"),
            (f"layers.{i}.gu_w", (2 * hc.base.ffn, H), "normal"), (f"layers.{i}.down_w", (H, hc.base.ffn), "normal")]


class HybridWeights:
    """Dense weights (embedding, attention layers, head) in the decoder's flat layout plus
    per-linear-layer tensors in a second flat buffer (fp32 conv taps / gates)."""

    def __init__(self, hc: HybridConfig, device, dtype=torch.bfloat16, seed: int = 0, std: float = 0.02,
                 grads: bool = True):
        """grads=False: frozen / serving weights (no gradient buffers, fp32 parameters without
        requires_grad)."""
        self.hc = hc
        cfg = hc.base
        self.layout = FlatLayout(cfg)
        grad_dt = torch.float64 if dtype == torch.float64 else torch.float32
        self.grad = torch.zeros(self.layout.total, dtype=grad_dt, device=device) if grads else None
        self.dense = Weights(cfg, init_flat(cfg, self.layout, device, dtype=dtype, seed=seed, std=std), self.layout,
                             self.grad)
        g = torch.Generator(device="cpu").manual_seed(seed + 11)
        self.t: dict[str, torch.Tensor] = {}
        self.fp32: dict[str, torch.Tensor] = {}
        for i in range(cfg.layers):
            if not hc.is_linear(i):
                continue
            for name, shape, init in _lin_specs(hc, i):
                if init == "ones":
                    w = torch.ones(shape, dtype=torch.float32)
                else:
                    w = torch.randn(shape, generator=g) * std
                    if init == "ba":
                        w[2 * hc.lin_heads:] = 0.0
                w = w.to(dtype).to(device)
                if grads:
                    w.main_grad = torch.zeros(shape, dtype=grad_dt, device=device)
                self.t[name] = w
            C = hc.lin_width
            pd = torch.float64 if dtype == torch.float64 else torch.float32
            for name, val in ((f"layers.{i}.conv_w", torch.randn(3 * C, hc.conv_width, generator=g) * 0.3),
                              (f"layers.{i}.A_log", torch.log(torch.rand(hc.lin_heads, generator=g) * 15 + 1)),
                              (f"layers.{i}.dt_bias", torch.randn(hc.lin_heads, generator=g) * 0.1)):
                self.fp32[name] = val.to(pd).to(device).requires_grad_(grads)

    def layer(self, i):
        return self.dense.layer(i)


def _rmsnorm_heads(o, w, eps):
    of = o.float()
    return (of * torch.rsqrt(of.pow(2).mean(-1, keepdim=True) + eps) * w.float()).to(o.dtype)


def linear_layer_forward(x, hw: HybridWeights, i: int, tree, lora=None):
    """One linear-recurrence layer over the tree rows x [T, H]; tree: (nodes [n, 4], tails [n, 8])."""
    hc, cfg = hw.hc, hw.hc.base
    t = hw.t
    nodes, tails = tree
    h = ops.rmsnorm(x, t[f"layers.{i}.ln1"], cfg.rms_eps, cfg.norm_plus_one)
    la = (lambda name: lora.get(f"layers.{i}.{name}")) if lora is not None else (lambda name: None)
    qkv = ops.linear(h, t[f"layers.{i}.lin_qkv"], lora=la("lin_qkv"))
    z = ops.linear(h, t[f"layers.{i}.lin_z"], lora=la("lin_z"))
    ba = ops.linear(h, t[f"layers.{i}.lin_ba"])  # [T, ba_rows]: beta logits | gate inputs | zero padding
    bb, aa = ba[:, :hc.lin_heads], ba[:, hc.lin_heads:2 * hc.lin_heads]
    W = hc.conv_width
    # conv context: the W - 1 rows before each node on its ancestor path (zeros when absent)
    rows = torch.as_tensor(tails[:, 8 - (W - 1):], device=x.device)
    ok = (rows >= 0).unsqueeze(-1)
    ctx = qkv.index_select(0, rows.clamp_min(0).reshape(-1)).view(len(nodes), W - 1, -1)
    cdt = torch.float64 if x.dtype == torch.float64 else torch.float32  # conv context: fp32 (exact for bf16)
    ctx = torch.where(ok, ctx.to(cdt), torch.zeros((), device=x.device, dtype=cdt))
    segs = [(int(s), int(e) - int(s)) for s, e, _, _ in nodes]
    qkv = causal_conv(qkv, hw.fp32[f"layers.{i}.conv_w"].to(cdt), None, segs, ctx=ctx,
                      ctx_idx=list(range(len(nodes))))
    C, Hh, d = hc.lin_width, hc.lin_heads, hc.lin_dim
    T = x.shape[0]
    q = torch.nn.functional.normalize(qkv[:, :C].float().view(T, Hh, d), dim=-1).to(x.dtype).reshape(T, C)
    k = torch.nn.functional.normalize(qkv[:, C:2 * C].float().view(T, Hh, d), dim=-1).to(x.dtype).reshape(T, C)
    v = qkv[:, 2 * C:].contiguous()
    gd = torch.float64 if x.dtype == torch.float64 else torch.float32
    beta = torch.sigmoid(bb.to(gd))
    g = -torch.exp(hw.fp32[f"layers.{i}.A_log"].to(gd)) * torch.nn.functional.softplus(
        aa.to(gd) + hw.fp32[f"layers.{i}.dt_bias"].to(gd))
    o = _tree_recurrence(q.contiguous(), k.contiguous(), v, g.contiguous(), beta.contiguous(), nodes,
                         d ** -0.5, hc.kind == "gdn")
    o = _rmsnorm_heads(o.view(T, Hh, d), t[f"layers.{i}.lin_norm"], cfg.rms_eps).reshape(T, C)
    o = (o.float() * torch.nn.functional.silu(z.float())).to(x.dtype)
    x = ops.linear(o, t[f"layers.{i}.lin_out"], None, residual=x, lora=la("lin_out"))
    h2 = ops.rmsnorm(x, t[f"layers.{i}.ln2"], cfg.rms_eps, cfg.norm_plus_one)
    act = ops.swiglu(ops.linear(h2, t[f"layers.{i}.gu_w"], lora=la("gu_w")))
    return ops.linear(act, t[f"layers.{i}.down_w"], None, residual=x, lora=la("down_w"))


def _tree_recurrence(q, k, v, g, beta, nodes, scale, delta):
    """Level-by-level recurrence: each node starts from its parent's final state."""
    depth = nodes[:, 3]
    out = torch.zeros_like(v)
    prev_fin, prev_index = None, {}
    for dlev in range(int(depth.max()) + 1 if len(nodes) else 0):
        ids = np.flatnonzero(depth == dlev)
        if not len(ids):
            continue
        rows = np.concatenate([np.arange(nodes[n, 0], nodes[n, 1]) for n in ids]).astype(np.int64)
        lens = [int(nodes[n, 1] - nodes[n, 0]) for n in ids]
        starts = np.r_[0, np.cumsum(lens)[:-1]]
        segs = list(zip(starts.tolist(), lens))
        ri = torch.as_tensor(rows, device=q.device)
        init_idx = [prev_index.get(int(nodes[n, 2]), -1) for n in ids] if prev_fin is not None else None
        o, fin = recurrence(q.index_select(0, ri), k.index_select(0, ri), v.index_select(0, ri),
                            g.index_select(0, ri), beta.index_select(0, ri), segs, scale, delta,
                            init_state=prev_fin, init_idx=init_idx)
        out = out.index_copy(0, ri, o)
        prev_fin, prev_index = fin, {int(n): j for j, n in enumerate(ids)}
    return out


def hybrid_forward(hw: HybridWeights, batch, temperature: float = 1.0, lora=None):
    """(logp, entropy) of the scored pairs of a prefix-tree micro-batch (TreeBatch with
    `nodes` / `path_tail`); lora: models.hybrid_lora.HybridLoRA adapters or None."""
    hc, cfg = hw.hc, hw.hc.base
    tree = (batch.nodes, batch.path_tail)
    x = ops.embed(batch.ids, hw.dense["embed"])
    if torch.is_grad_enabled() and not x.requires_grad:
        x.requires_grad_(True)  # a graph even when only adapters (plain tensors with main_grad) train
    for i in range(cfg.layers):
        if hc.is_linear(i):
            x = linear_layer_forward(x, hw, i, tree, lora)
        else:
            x = layer_forward(x, hw.layer(i), cfg, batch.pos, batch.plan, lora.layer(i) if lora is not None else None)
    hf = ops.rmsnorm(x, hw.dense["norm"], cfg.rms_eps, cfg.norm_plus_one)
    hp = hf.index_select(0, batch.pair_rows)
    return ops.logprob_head(hp, hw.dense.head, batch.pair_labels, 1.0 / temperature, cfg.vocab_size)


__all__ = ["FAMILIES", "HybridConfig", "HybridWeights", "family_kind", "hybrid_config", "hybrid_forward",
           "linear_layer_forward"]
