"""Model configurations (dense Qwen2.5-family shapes and the tiny test decoder).

The architecture is the Qwen2 decoder: RMSNorm -> fused QKV (+bias) -> RoPE ->
GQA attention -> O proj (+residual) -> RMSNorm -> fused gate/up -> SwiGLU -> down
proj (+residual); final RMSNorm and an LM head (optionally tied to the embedding).
"""
from __future__ import annotations

from dataclasses import asdict, dataclass, replace


@dataclass(frozen=True)
class ModelConfig:
    name: str
    vocab_size: int
    hidden: int
    layers: int
    heads: int
    kv_heads: int
    head_dim: int
    ffn: int
    rope_theta: float = 1_000_000.0
    rms_eps: float = 1e-6
    qkv_bias: bool = True
    tie_embeddings: bool = False
    norm_plus_one: bool = False  # Qwen3.5-style (1 + w) norms
    max_position: int = 131072

    @property
    def qkv_width(self) -> int:
        return (self.heads + 2 * self.kv_heads) * self.head_dim

    @property
    def q_width(self) -> int:
        return self.heads * self.head_dim

    @property
    def kv_width(self) -> int:
        return self.kv_heads * self.head_dim

    def num_params(self) -> int:
        H, F = self.hidden, self.ffn
        per_layer = 2 * H + self.qkv_width * H + (self.qkv_width if self.qkv_bias else 0) + H * self.q_width \
            + 2 * F * H + H * F
        emb = self.vocab_size * H
        return self.layers * per_layer + H + emb * (1 if self.tie_embeddings else 2)

    def flops_per_token(self, ctx: float = 0.0) -> float:
        """Forward matmul FLOPs per token (2 * non-embedding params + head) + attention."""
        H, F = self.hidden, self.ffn
        lin = self.qkv_width * H + H * self.q_width + 3 * F * H
        attn = 2 * self.q_width * ctx  # QK^T and PV, per token per layer (x2 flops/mac folded below)
        return 2.0 * (self.layers * lin + self.vocab_size * H) + 2.0 * self.layers * attn

    def to_dict(self):
        return asdict(self)

    def with_(self, **kw) -> "ModelConfig":
        return replace(self, **kw)


PRESETS = {
    # tiny random-init decoder for exactness tests
    "tiny": ModelConfig("tiny", vocab_size=4096, hidden=256, layers=2, heads=4, kv_heads=4, head_dim=64, ffn=688,
                        rope_theta=10000.0, qkv_bias=False),
    # small GQA decoder with head_dim 128 for the tensor-parallel engine tests (tp <= 4)
    "tiny-tp": ModelConfig("tiny-tp", vocab_size=4096, hidden=512, layers=2, heads=8, kv_heads=4, head_dim=128,
                           ffn=1024, rope_theta=10000.0),
    "qwen2.5-1.5b": ModelConfig("qwen2.5-1.5b", vocab_size=151936, hidden=1536, layers=28, heads=12, kv_heads=2,
                                head_dim=128, ffn=8960, tie_embeddings=True),
    "qwen2.5-7b": ModelConfig("qwen2.5-7b", vocab_size=152064, hidden=3584, layers=28, heads=28, kv_heads=4,
                              head_dim=128, ffn=18944),
    "qwen2.5-32b": ModelConfig("qwen2.5-32b", vocab_size=152064, hidden=5120, layers=64, heads=40, kv_heads=8,
                               head_dim=128, ffn=27648, rms_eps=1e-5),
}


def get_config(name: str, **overrides) -> ModelConfig:
    cfg = PRESETS[name]
    return cfg.with_(**overrides) if overrides else cfg
