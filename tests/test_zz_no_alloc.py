"""The allocation-free decode attention entry point, called through its exported C symbol.

Callers that cannot allocate device memory (a runtime that owns all GPU memory, a
fixed-budget serving loop, a loop that cannot afford an allocation's implicit sync)
use `octo_decode_attention_noalloc`; it must give the same result as the regular
decode path, on consecutive calls that reuse its static scratch.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    import octopus_b200._C as C

    lib = ctypes.CDLL(C.__file__)
    fn = lib.octo_decode_attention_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 7 + [ctypes.c_int] * 7 + [ctypes.c_float, ctypes.c_void_p]
    return fn


def _case(seed, B, Hq, Hkv, D, slots=5000, max_len=1200):
    g = torch.Generator().manual_seed(seed)
    dev = "cuda"
    kc = torch.randn(slots, Hkv * D, generator=g).bfloat16().to(dev)
    vc = torch.randn(slots, Hkv * D, generator=g).bfloat16().to(dev)
    lens = torch.randint(1, max_len, (B,), generator=g, dtype=torch.int32)
    start = torch.zeros(B, dtype=torch.int32)
    start[1:] = torch.cumsum(lens, 0)[:-1]
    idx = torch.randint(0, slots, (int(lens.sum()),), generator=g, dtype=torch.int32)
    q = torch.randn(B, Hq * D, generator=g).bfloat16().to(dev)
    return q, kc, vc, start.to(dev), lens.to(dev), idx.to(dev)


def _rel(a, b):
    return float((a.float() - b.float()).norm() / (b.float().norm() + 1e-12))


def test_noalloc_matches_regular_decode_two_calls():
    from octopus_b200 import ops

    fn = _lib()
    stream = torch.cuda.current_stream()
    for seed, (B, Hq, Hkv, D, splits) in enumerate([(37, 28, 4, 128, 8), (19, 12, 2, 128, 4)]):
        q, kc, vc, start, lens, idx = _case(seed, B, Hq, Hkv, D)
        ref = ops.DecodeAttention(Hq, Hkv, D, B, splits, "cuda")(q, kc, vc, start, idx, kv_len=lens)
        out = torch.empty_like(q)
        rc = fn(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), start.data_ptr(), lens.data_ptr(), idx.data_ptr(),
                out.data_ptr(), B, Hq, Hkv, D, q.stride(0), out.stride(0), splits, D ** -0.5, stream.cuda_stream)
        torch.cuda.synchronize()
        assert rc == 0
        assert _rel(out, ref) < 2e-2


def test_noalloc_rejects_sizes_beyond_its_scratch():
    fn = _lib()
    B, Hq, Hkv, D, splits = 4096, 32, 8, 128, 64  # 4096*32*64*128 floats >> the static limit
    rc = fn(0, 0, 0, 0, 0, 0, 0, B, Hq, Hkv, D, Hq * D, Hq * D, splits, 0.1, torch.cuda.current_stream().cuda_stream)
    assert rc == -1
