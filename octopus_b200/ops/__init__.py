"""sm_100a kernels (CUDA tensors) with plain-PyTorch references (CPU tensors)."""
from ._ext import (KernelError, add_launches, available, check_status, ext, launches, pdl_launches, read_status,
                   set_wait_budget, wait_budget)
from .core import (AttnPlan, adamw_, attention, attention_kv, embed, gemm, gemm_swiglu, linear, linear_rope, logprob_head, rmsnorm,
                   rope_, sample, sqnorm_, swiglu)
from .decode import DecodeAttention, SharedDecode, decode_attention

__all__ = [
    "AttnPlan", "DecodeAttention", "SharedDecode", "adamw_", "add_launches", "launches", "attention", "attention_kv", "available", "check_status", "decode_attention", "embed",
    "ext", "gemm", "gemm_swiglu", "linear_rope", "pdl_launches", "KernelError", "read_status", "set_wait_budget", "wait_budget", "linear", "logprob_head", "rmsnorm", "rope_", "sample", "sqnorm_", "swiglu",
]
