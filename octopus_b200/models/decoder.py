"""Dense decoder (Qwen2 family) over flat parameter buffers.

All parameters live in one flat bf16 buffer, grouped into *units* (embedding, one per
decoder layer, final norm + head).  Units are contiguous and padded so that the FSDP
actor can shard every unit evenly; single-GPU training uses the same layout.  Each
parameter tensor is a view into the flat buffer and carries an fp32 ``main_grad``
view into a flat fp32 gradient buffer, which the wgrad GEMM epilogues accumulate
into directly.

Training forward (`forward_tree`) runs one prefix-tree micro-batch: every tree row
once, tree attention over gathered key lists, per-layer activation checkpointing,
and the chunked logprob head over (row, label) pairs.  Reference parity:
`octopus/rl/prefix_tree.py:381-446` (tree forward), `octopus/rl/seq_tiles.py:207-234`
(layer forward), `octopus/rl/lm_head.py:115-153` (head over scored rows).

Checkpoints are HF-layout safetensors (`model.layers.{i}.self_attn.q_proj.weight`, ...);
`octopus/rl/text_checkpoint.py:1-56` is the reference's converter to that layout.
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass

import torch

from .. import ops
from .config import ModelConfig

ALIGN = 256  # elements; every parameter view starts 512-byte aligned (TMA needs 16)


@dataclass
class Spec:
    name: str
    shape: tuple
    unit: int
    init: str  # "normal" | "ones" | "zeros"


def param_specs(cfg: ModelConfig) -> list[Spec]:
    H, F = cfg.hidden, cfg.ffn
    specs = [Spec("embed", (cfg.vocab_size, H), 0, "normal")]
    for i in range(cfg.layers):
        u = i + 1
        specs += [
            Spec(f"layers.{i}.ln1", (H,), u, "ones"),
            Spec(f"layers.{i}.qkv_w", (cfg.qkv_width, H), u, "normal"),
        ]
        if cfg.qkv_bias:
            specs.append(Spec(f"layers.{i}.qkv_b", (cfg.qkv_width,), u, "zeros"))
        specs += [
            Spec(f"layers.{i}.o_w", (H, cfg.q_width), u, "normal"),
            Spec(f"layers.{i}.ln2", (H,), u, "ones"),
            Spec(f"layers.{i}.gu_w", (2 * F, H), u, "normal"),
            Spec(f"layers.{i}.down_w", (H, F), u, "normal"),
        ]
    last = cfg.layers + 1
    specs.append(Spec("norm", (H,), last, "ones"))
    if not cfg.tie_embeddings:
        specs.append(Spec("lm_head", (cfg.vocab_size, H), last, "normal"))
    return specs


def _round(n: int, a: int) -> int:
    return (n + a - 1) // a * a


class FlatLayout:
    """Offsets of every parameter in the flat buffer; units padded to `pad_multiple`."""

    def __init__(self, cfg: ModelConfig, pad_multiple: int = 1):
        self.cfg = cfg
        self.specs = param_specs(cfg)
        self.offsets: dict[str, int] = {}
        self.units: list[tuple[int, int]] = []
        unit_align = ALIGN * max(1, pad_multiple)
        off = 0
        cur_unit = -1
        unit_start = 0
        for s in self.specs:
            if s.unit != cur_unit:
                if cur_unit >= 0:
                    end = _round(off, unit_align)
                    self.units.append((unit_start, end))
                    off = end
                cur_unit = s.unit
                unit_start = off
            off = _round(off, ALIGN)
            self.offsets[s.name] = off
            off += math.prod(s.shape)
        end = _round(off, unit_align)
        self.units.append((unit_start, end))
        self.total = end
        self.unit_of = {s.name: s.unit for s in self.specs}
        self.shape_of = {s.name: s.shape for s in self.specs}

    def numel(self, name):
        return math.prod(self.shape_of[name])


class Weights:
    """Views of the model parameters into a flat bf16 buffer (and fp32 grads)."""

    def __init__(self, cfg: ModelConfig, flat: torch.Tensor, layout: FlatLayout, grad: torch.Tensor | None = None):
        self.cfg, self.flat, self.layout = cfg, flat, layout
        self.t: dict[str, torch.Tensor] = {}
        for s in layout.specs:
            o = layout.offsets[s.name]
            v = flat[o: o + math.prod(s.shape)].view(s.shape)
            if grad is not None:
                v.main_grad = grad[o: o + math.prod(s.shape)].view(s.shape)
            self.t[s.name] = v

    def __getitem__(self, k):
        return self.t[k]

    @property
    def head(self) -> torch.Tensor:
        return self.t["embed"] if self.cfg.tie_embeddings else self.t["lm_head"]

    def layer(self, i):
        c = self.cfg
        g = self.t.get
        return (g(f"layers.{i}.ln1"), g(f"layers.{i}.qkv_w"), g(f"layers.{i}.qkv_b"), g(f"layers.{i}.o_w"),
                g(f"layers.{i}.ln2"), g(f"layers.{i}.gu_w"), g(f"layers.{i}.down_w"))


def init_flat(cfg: ModelConfig, layout: FlatLayout, device, dtype=torch.bfloat16, seed: int = 0,
              std: float = 0.02) -> torch.Tensor:
    """Random-init flat parameters (normal(0, std) matrices, unit norms, zero biases)."""
    flat = torch.zeros(layout.total, dtype=dtype, device=device)
    gen = torch.Generator(device=device).manual_seed(seed)
    for s in layout.specs:
        o = layout.offsets[s.name]
        n = math.prod(s.shape)
        if s.init == "normal":
            flat[o: o + n].normal_(0.0, std, generator=gen)
        elif s.init == "ones":
            flat[o: o + n].fill_(0.0 if cfg.norm_plus_one else 1.0)
    return flat


# ----------------------------------------------------------------------------- forward
@dataclass
class TreeBatch:
    """One prefix-tree micro-batch on device (see octopus_b200.rl.prefix_tree)."""

    ids: torch.Tensor        # [T] int64 tree-row tokens (T padded to a multiple of 128)
    pos: torch.Tensor        # [T] int32 K2 positions
    plan: ops.AttnPlan       # attention over gathered key lists
    pair_rows: torch.Tensor  # [M] int64 rows whose next-token logprob is scored
    pair_labels: torch.Tensor  # [M] int64 label of each pair


def qkv_rope(h, qkv_w, qkv_b, pos, cfg: ModelConfig, lora=None):
    """The fused q / k / v projection with the rotary embedding on q and k: one GEMM with
    the rotation in its epilogue, or (LoRA adapters) the projection, then rope_."""
    if lora is None:
        return ops.linear_rope(h, qkv_w, qkv_b, pos, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.rope_theta)
    qkv = ops.linear(h, qkv_w, qkv_b, lora=lora)
    return ops.rope_(qkv, pos, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.rope_theta)


def layer_forward(x, w, cfg: ModelConfig, pos, plan, lw=None):
    """One decoder layer; lw: the layer's LoRA adapters (qkv, o, gu, down), each
    (A, B, scale) or None."""
    ln1, qkv_w, qkv_b, o_w, ln2, gu_w, down_w = w
    la = lw if lw is not None else (None, None, None, None)
    h = ops.rmsnorm(x, ln1, cfg.rms_eps, cfg.norm_plus_one)
    qkv = qkv_rope(h, qkv_w, qkv_b, pos, cfg, la[0])
    a = ops.attention(qkv, plan, cfg.heads, cfg.kv_heads, cfg.head_dim)
    x = ops.linear(a, o_w, None, residual=x, lora=la[1])
    h2 = ops.rmsnorm(x, ln2, cfg.rms_eps, cfg.norm_plus_one)
    act = _mlp_act(h2, gu_w, la[2])
    return ops.linear(act, down_w, None, residual=x, lora=la[3])


def _mlp_act(h2, gu_w, lora):
    """swiglu(h2 gu_w^T): without autograd (checkpointed forwards) one GEMM with the
    activation in its epilogue; with autograd the projection is kept for the backward."""
    if lora is None and not torch.is_grad_enabled():
        return ops.gemm_swiglu(h2, gu_w)
    return ops.swiglu(ops.linear(h2, gu_w, lora=lora))


def _mlp_part(x, a, w, cfg, lw):
    """The row-wise rest of a layer after attention: o-projection + residual, RMSNorm,
    SwiGLU MLP + residual."""
    _, _, _, o_w, ln2, gu_w, down_w = w
    la = lw if lw is not None else (None, None, None, None)
    x = ops.linear(a, o_w, None, residual=x, lora=la[1])
    h2 = ops.rmsnorm(x, ln2, cfg.rms_eps, cfg.norm_plus_one)
    act = _mlp_act(h2, gu_w, la[2])
    return ops.linear(act, down_w, None, residual=x, lora=la[3])


class _TileCkpt(torch.autograd.Function):
    """Checkpoint of _mlp_part on one row tile (inputs x, a): backward recomputes the tile,
    so only one tile's MLP activations exist at a time."""

    @staticmethod
    def forward(ctx, x, a, w, cfg, lw):
        ctx.args = (w, cfg, lw)
        ctx.save_for_backward(x, a)
        with torch.no_grad():
            return _mlp_part(x, a, w, cfg, lw)

    @staticmethod
    def backward(ctx, dy):
        x, a = ctx.saved_tensors
        xr, ar = x.detach().requires_grad_(True), a.detach().requires_grad_(True)
        with torch.enable_grad():
            y = _mlp_part(xr, ar, *ctx.args)
        torch.autograd.backward(y, dy)
        return xr.grad, ar.grad, None, None, None


def layer_forward_tiled(x, w, cfg: ModelConfig, pos, plan, lw=None, tile: int = 16384):
    """layer_forward with the row-wise part in tiles of `tile` rows, each checkpointed: the
    q / k / v projection and attention see the whole tree (keys come from any row), the
    o-projection and MLP run tile by tile, so their activations follow the tile, not the
    tree."""
    ln1, qkv_w, qkv_b = w[0], w[1], w[2]
    la = lw if lw is not None else (None, None, None, None)
    h = ops.rmsnorm(x, ln1, cfg.rms_eps, cfg.norm_plus_one)
    qkv = qkv_rope(h, qkv_w, qkv_b, pos, cfg, la[0])
    a = ops.attention(qkv, plan, cfg.heads, cfg.kv_heads, cfg.head_dim)
    T = x.shape[0]
    tile = max(8, tile // 8 * 8)
    if T <= tile:
        return _mlp_part(x, a, w, cfg, lw)
    outs = []
    for r0 in range(0, T, tile):
        xt, at = x[r0:r0 + tile], a[r0:r0 + tile]
        outs.append(_TileCkpt.apply(xt, at, w, cfg, lw) if torch.is_grad_enabled() else _mlp_part(xt, at, w, cfg, lw))
    return torch.cat(outs)


class _Ckpt(torch.autograd.Function):
    """Activation checkpoint of fn(x, *args): forward without a graph, the input saved
    through autograd's saved-tensor hooks (so host-resident activations apply to it),
    recompute with a graph in backward.  Weight gradients accumulate into main_grad
    inside the recompute's backward."""

    @staticmethod
    def forward(ctx, x, fn, *args):
        ctx.fn, ctx.args = fn, args
        ctx.save_for_backward(x)
        with torch.no_grad():
            return fn(x, *args)

    @staticmethod
    def backward(ctx, dy):
        (x,) = ctx.saved_tensors
        xr = x.detach().requires_grad_(True)
        with torch.enable_grad():
            y = ctx.fn(xr, *ctx.args)
        torch.autograd.backward(y, dy)
        return (xr.grad, None) + (None,) * len(ctx.args)


def _layers_forward(x, ws, cfg, pos, plan, lws, lf=layer_forward):
    """Several layers (a checkpoint block); during the block's recompute each layer is
    checkpointed again, so backward holds one layer's working set at a time."""
    for w, lw in zip(ws, lws):
        x = _Ckpt.apply(x, lf, w, cfg, pos, plan, lw) if torch.is_grad_enabled() else lf(x, w, cfg, pos, plan, lw)
    return x


def forward_tree(weights: Weights, batch: TreeBatch, temperature: float = 1.0, ckpt: bool = True,
                 layer_hook=None, ckpt_block: int = 1, lora=None, seq_tile: int = 0):
    """Returns (logp [M], entropy [M]) of the scored (row, label) pairs.

    ckpt: activation checkpointing; ckpt_block = k keeps only every k-th layer input
    (block checkpoint: the inputs of the layers inside a block are recomputed); seq_tile > 0:
    each layer's o-projection and MLP run in checkpointed tiles of that many rows
    (layer_forward_tiled)."""
    cfg = weights.cfg
    if seq_tile and seq_tile < batch.ids.shape[0]:
        lf = lambda *a: layer_forward_tiled(*a, tile=seq_tile)  # noqa: E731
    else:
        lf = layer_forward
    x = ops.embed(batch.ids, weights["embed"])
    if x.requires_grad is False and torch.is_grad_enabled():
        x.requires_grad_(True)
    if ckpt and ckpt_block > 1 and torch.is_grad_enabled() and layer_hook is None:
        for i0 in range(0, cfg.layers, ckpt_block):
            idx = range(i0, min(cfg.layers, i0 + ckpt_block))
            ws = [weights.layer(i) for i in idx]
            lws = [lora.layer(i) if lora is not None else None for i in idx]
            x = _Ckpt.apply(x, _layers_forward, ws, cfg, batch.pos, batch.plan, lws, lf)
        h = ops.rmsnorm(x, weights["norm"], cfg.rms_eps, cfg.norm_plus_one)
        hp = h.index_select(0, batch.pair_rows)
        return ops.logprob_head(hp, weights.head, batch.pair_labels, 1.0 / temperature, cfg.vocab_size)
    for i in range(cfg.layers):
        if layer_hook is not None:
            layer_hook(i)
        w = weights.layer(i)
        lw = lora.layer(i) if lora is not None else None
        if ckpt and torch.is_grad_enabled():
            x = _Ckpt.apply(x, lf, w, cfg, batch.pos, batch.plan, lw)
        else:
            x = lf(x, w, cfg, batch.pos, batch.plan, lw)
    if layer_hook is not None:
        layer_hook(cfg.layers)
    h = ops.rmsnorm(x, weights["norm"], cfg.rms_eps, cfg.norm_plus_one)
    hp = h.index_select(0, batch.pair_rows)
    return ops.logprob_head(hp, weights.head, batch.pair_labels, 1.0 / temperature, cfg.vocab_size)


# ----------------------------------------------------------------------------- HF checkpoints
def hf_tensors(weights: Weights) -> dict[str, torch.Tensor]:
    """Split fused tensors into HF Qwen2 names (views, no copies where possible)."""
    cfg = weights.cfg
    q, kv = cfg.q_width, cfg.kv_width
    F = cfg.ffn
    out = {"model.embed_tokens.weight": weights["embed"], "model.norm.weight": weights["norm"]}
    if not cfg.tie_embeddings:
        out["lm_head.weight"] = weights["lm_head"]
    for i in range(cfg.layers):
        p = f"model.layers.{i}."
        qkv_w = weights[f"layers.{i}.qkv_w"]
        out[p + "input_layernorm.weight"] = weights[f"layers.{i}.ln1"]
        out[p + "self_attn.q_proj.weight"] = qkv_w[:q]
        out[p + "self_attn.k_proj.weight"] = qkv_w[q: q + kv]
        out[p + "self_attn.v_proj.weight"] = qkv_w[q + kv:]
        if cfg.qkv_bias:
            b = weights[f"layers.{i}.qkv_b"]
            out[p + "self_attn.q_proj.bias"] = b[:q]
            out[p + "self_attn.k_proj.bias"] = b[q: q + kv]
            out[p + "self_attn.v_proj.bias"] = b[q + kv:]
        out[p + "self_attn.o_proj.weight"] = weights[f"layers.{i}.o_w"]
        out[p + "post_attention_layernorm.weight"] = weights[f"layers.{i}.ln2"]
        gu = weights[f"layers.{i}.gu_w"]
        out[p + "mlp.gate_proj.weight"] = gu[:F]
        out[p + "mlp.up_proj.weight"] = gu[F:]
        out[p + "mlp.down_proj.weight"] = weights[f"layers.{i}.down_w"]
    return out


def save_hf(weights: Weights, path: str, max_shard_bytes: int = 5 << 30) -> list[str]:
    """Write HF-layout safetensors shards + index + config.json."""
    import json

    from safetensors.torch import save_file

    os.makedirs(path, exist_ok=True)
    tensors = {k: v.detach().contiguous().cpu() for k, v in hf_tensors(weights).items()}
    shards, cur, size = [], {}, 0
    for k, v in tensors.items():
        nb = v.numel() * v.element_size()
        if cur and size + nb > max_shard_bytes:
            shards.append(cur)
            cur, size = {}, 0
        cur[k] = v
        size += nb
    if cur:
        shards.append(cur)
    names, index = [], {}
    for i, sh in enumerate(shards):
        fn = f"model-{i + 1:05d}-of-{len(shards):05d}.safetensors"
        save_file(sh, os.path.join(path, fn), metadata={"format": "pt"})
        names.append(fn)
        for k in sh:
            index[k] = fn
    with open(os.path.join(path, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {"total_size": sum(v.numel() * v.element_size() for v in tensors.values())},
                   "weight_map": index}, f, indent=1)
    cfg = weights.cfg
    hf_cfg = {
        "architectures": ["Qwen2ForCausalLM"], "model_type": "qwen2", "vocab_size": cfg.vocab_size,
        "hidden_size": cfg.hidden, "num_hidden_layers": cfg.layers, "num_attention_heads": cfg.heads,
        "num_key_value_heads": cfg.kv_heads, "intermediate_size": cfg.ffn, "rope_theta": cfg.rope_theta,
        "rms_norm_eps": cfg.rms_eps, "tie_word_embeddings": cfg.tie_embeddings, "torch_dtype": "bfloat16",
        "hidden_act": "silu", "max_position_embeddings": cfg.max_position, "head_dim": cfg.head_dim,
    }
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(hf_cfg, f, indent=1)
    return names


def load_hf(weights: Weights, path: str) -> None:
    """Load HF-layout safetensors into the flat views (in place)."""
    import glob

    from safetensors import safe_open

    targets = hf_tensors(weights)
    seen = set()
    for fn in sorted(glob.glob(os.path.join(path, "*.safetensors"))):
        with safe_open(fn, framework="pt") as f:
            for k in f.keys():
                if k in targets:
                    with torch.no_grad():
                        targets[k].copy_(f.get_tensor(k).to(targets[k].dtype))
                    seen.add(k)
    missing = set(targets) - seen
    if missing:
        raise KeyError(f"checkpoint at {path} misses {sorted(missing)[:5]} ...")
