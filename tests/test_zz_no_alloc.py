"""The allocation-free decode attention entry point, called through its exported C symbol.

Some callers cannot allocate device memory while they run: a plugin inside a runtime
that owns all of the GPU's memory, a serving loop with a memory budget fixed up front,
or a latency-critical loop that cannot afford the implicit synchronisation of an
allocation.  They call `octo_decode_attention_noalloc`, whose split-K scratch is a
static device array.  It must give the regular decode path's result (and a plain fp32
attention's, within bf16 tolerance) on consecutive calls that reuse that scratch, and
it must take no device memory from the PyTorch allocator.
"""
import ctypes
import gc

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


def _case(seed, B, Hq, Hkv, D, dev, slots=5000, max_len=1200, short_rows=0):
    g = torch.Generator().manual_seed(seed)
    kc = torch.randn(slots, Hkv * D, generator=g).bfloat16().to(dev)
    vc = torch.randn(slots, Hkv * D, generator=g).bfloat16().to(dev)
    lens = torch.randint(1, max_len, (B,), generator=g, dtype=torch.int32)
    lens[:short_rows] = 1  # single-key rows: most splits of these rows are empty
    start = torch.zeros(B, dtype=torch.int32)
    start[1:] = torch.cumsum(lens, 0)[:-1]
    idx = torch.randint(0, slots, (int(lens.sum()),), generator=g, dtype=torch.int32)
    q = torch.randn(B, Hq * D, generator=g).bfloat16().to(dev)
    return q, kc, vc, start.to(dev), lens.to(dev), idx.to(dev)


def _fp32_reference(q, kc, vc, start, lens, idx, Hq, Hkv, D):
    G = Hq // Hkv
    out = torch.empty(q.shape, dtype=torch.float32, device=q.device)
    for b in range(q.shape[0]):
        s, n = int(start[b]), int(lens[b])
        rows = idx[s: s + n].long()
        k = kc[rows].float().view(n, Hkv, D).repeat_interleave(G, dim=1)  # [n, Hq, D]
        v = vc[rows].float().view(n, Hkv, D).repeat_interleave(G, dim=1)
        qb = q[b].float().view(Hq, D)
        p = torch.softmax(torch.einsum("hd,nhd->hn", qb, k) * D ** -0.5, dim=-1)
        out[b] = torch.einsum("hn,nhd->hd", p, v).reshape(-1)
    return out


def _rel(a, b):
    return float((a.float() - b.float()).norm() / (b.float().norm() + 1e-12))


def _call(fn, q, kc, vc, start, lens, idx, out, Hq, Hkv, D, splits):
    return fn(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), start.data_ptr(), lens.data_ptr(), idx.data_ptr(),
              out.data_ptr(), q.shape[0], Hq, Hkv, D, q.stride(0), out.stride(0), splits, D ** -0.5,
              torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("splits", [1, 2, 64])
def test_noalloc_matches_regular_decode_two_calls(D, splits):
    from octopus_b200 import ops

    fn = _lib()
    dev = torch.device("cuda", 0)
    # the second call uses a larger B * Hq * splits footprint than the first, as large as
    # the static scratch allows (2 Mi partial floats) up to 37 rows
    big = min(37, (2 * 1024 * 1024) // (28 * splits * D))
    for seed, (B, Hq, Hkv) in enumerate([(min(9, big), 12, 2), (big, 28, 4)]):
        q, kc, vc, start, lens, idx = _case(seed + 10 * D + splits, B, Hq, Hkv, D, dev, short_rows=3)
        ref32 = _fp32_reference(q, kc, vc, start, lens, idx, Hq, Hkv, D)
        ref = ops.DecodeAttention(Hq, Hkv, D, B, splits, dev)(q, kc, vc, start, idx, kv_len=lens)
        out = torch.empty_like(q)
        # (earlier tests' tensors held in reference cycles must not be collected while the
        # counters are compared: collect them now and keep the collector off meanwhile)
        gc.collect()
        gc.disable()
        try:
            torch.cuda.synchronize()
            alloc, reserved = torch.cuda.memory_allocated(dev), torch.cuda.memory_reserved(dev)
            rc = _call(fn, q, kc, vc, start, lens, idx, out, Hq, Hkv, D, splits)
            torch.cuda.synchronize()
            after = torch.cuda.memory_allocated(dev), torch.cuda.memory_reserved(dev)
        finally:
            gc.enable()
        assert rc == 0
        assert after == (alloc, reserved)
        assert _rel(out, ref) < 2e-2
        assert _rel(out, ref32) < 2e-2


def test_noalloc_on_a_second_device():
    """The scratch address and the kernels' shared-memory opt-in are per device."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    fn = _lib()
    for d in (0, 1):
        dev = torch.device("cuda", d)
        with torch.cuda.device(dev):
            q, kc, vc, start, lens, idx = _case(d, 11, 28, 4, 128, dev)
            ref32 = _fp32_reference(q, kc, vc, start, lens, idx, 28, 4, 128)
            out = torch.empty_like(q)
            assert _call(fn, q, kc, vc, start, lens, idx, out, 28, 4, 128, 8) == 0
            torch.cuda.synchronize(dev)
            assert _rel(out, ref32) < 2e-2


def test_noalloc_rejects_sizes_beyond_its_scratch():
    fn = _lib()
    B, Hq, Hkv, D, splits = 4096, 32, 8, 128, 64  # 4096*32*64*128 floats >> the static limit
    rc = fn(0, 0, 0, 0, 0, 0, 0, B, Hq, Hkv, D, Hq * D, Hq * D, splits, 0.1, torch.cuda.current_stream().cuda_stream)
    assert rc == -1


def test_noalloc_rejects_misaligned_inputs():
    fn = _lib()
    dev = torch.device("cuda", 0)
    q, kc, vc, start, lens, idx = _case(3, 4, 8, 2, 64, dev)
    out = torch.empty_like(q)
    base = (q.data_ptr(), kc.data_ptr(), vc.data_ptr(), start.data_ptr(), lens.data_ptr(), idx.data_ptr(),
            out.data_ptr())
    st = torch.cuda.current_stream().cuda_stream
    bad_k = list(base)
    bad_k[1] += 2  # K cache not 16-byte aligned
    assert fn(*bad_k, 4, 8, 2, 64, 512, 512, 2, 0.125, st) == -2
    assert fn(*base, 4, 8, 2, 64, 511, 512, 2, 0.125, st) == -2  # ldq below Hq * head_dim
    assert fn(*base, 4, 8, 2, 64, 512, 512, 2, 0.125, st) == 0
    torch.cuda.synchronize()
