"""Micro-benchmarks of the sm_100a kernels against cuBLAS / plain PyTorch.

    python -m octopus_b200.tools.bench_kernels [--shapes 7b] [--json out.json]

Times each kernel with CUDA events after warm-up (median of repeats); inputs of the
GEMM shapes are larger than L2 for the big cases.  Reports TFLOP/s (GEMM-like) or
GB/s (memory-bound) and the fraction of MEASURED_PEAKS.json when it is present.
"""
from __future__ import annotations

import argparse
import json
import os

import numpy as np
import torch

from octopus_b200 import ops


def timeit(fn, warmup=3, reps=10):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(reps):
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b))
    return float(np.median(ts))


def peaks():
    p = os.path.join(os.path.dirname(__file__), "..", "..", "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return json.load(f)
    except OSError:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def gemm_cases(kind):
    if kind == "7b":
        T, H, F, Wqkv = 16384, 3584, 18944, 4608
        return [("qkv_fwd", T, Wqkv, H, False, False), ("o_fwd", T, H, H, False, False),
                ("gate_up_fwd", T, 2 * F, H, False, False), ("down_fwd", T, H, F, False, False),
                ("gate_up_dgrad", T, H, 2 * F, False, True), ("gate_up_wgrad", 2 * F, H, T, True, True),
                ("down_dgrad", T, F, H, False, True), ("down_wgrad", H, F, T, True, True),
                ("decode_qkv_b256", 256, Wqkv, H, False, False), ("decode_gate_up_b256", 256, 2 * F, H, False, False),
                ("square_8192", 8192, 8192, 8192, False, False)]
    return [("square_4096", 4096, 4096, 4096, False, False)]


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--shapes", default="7b")
    ap.add_argument("--json", default=None)
    args = ap.parse_args(argv)
    pk = peaks()
    res = []
    dev = "cuda"
    for name, M, N, K, a_mn, b_mn in gemm_cases(args.shapes):
        A = torch.randn(K, M, device=dev).bfloat16() if a_mn else torch.randn(M, K, device=dev).bfloat16()
        B = torch.randn(K, N, device=dev).bfloat16() if b_mn else torch.randn(N, K, device=dev).bfloat16()
        C = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
        t = timeit(lambda: ops.gemm(A, B, a_mn=a_mn, b_mn=b_mn, out=C))
        At = A.t() if a_mn else A
        Bt = B if b_mn else B.t()
        tc = timeit(lambda: torch.matmul(At, Bt, out=C))
        fl = 2.0 * M * N * K
        r = {"kernel": "gemm_tcgen05", "case": name, "M": M, "N": N, "K": K, "ms": t, "tflops": fl / t / 1e9,
             "cublas_ms": tc, "cublas_tflops": fl / tc / 1e9, "frac_of_measured": fl / t / 1e9 / pk["bf16_tflops"]}
        res.append(r)
        print(json.dumps(r), flush=True)
    ops.check_status(0)
    # tree attention fwd+bwd: 7B heads, 8 sequences sharing a 2048 prefix + 2048 own tokens
    Hq, Hkv, D = 28, 4, 128
    pre, own, nseq = 2048, 2048, 8
    T = pre + nseq * own
    cu_q, cu_k, keys = [0, pre], [0, pre], list(range(pre))
    for s in range(nseq):
        a = pre + s * own
        cu_q.append(cu_q[-1] + own)
        keys += list(range(pre)) + list(range(a, a + own))
        cu_k.append(len(keys))
    plan = ops.AttnPlan.build(cu_q, cu_k, np.asarray(keys, dtype=np.int32), dev)
    qkv = (torch.randn(T, (Hq + 2 * Hkv) * D, device=dev) * 0.5).bfloat16()
    pairs = pre * (pre + 1) / 2 + nseq * (own * pre + own * (own + 1) / 2)
    fl = 4.0 * pairs * Hq * D
    q, k, v = qkv[:, : Hq * D], qkv[:, Hq * D: (Hq + Hkv) * D], qkv[:, (Hq + Hkv) * D:]
    for tc in (0, 2):  # mma.sync (the head_dim != 128 path) for comparison, tcgen05
        t = timeit(lambda: ops.ext().attn_fwd(q, k, v, plan.cu_q, plan.cu_k, plan.key_idx, plan.tiles_for(tc), Hq, Hkv,
                                              D, D ** -0.5, True, True, tc))
        name = {0: "tree_attn_fwd_mma_sync", 2: "tree_attn_fwd_tcgen05_2tile"}[tc]
        r = {"kernel": name, "T": T, "ms": t,
             "tflops": fl / t / 1e9, "frac_of_measured": fl / t / 1e9 / pk["bf16_tflops"]}
        res.append(r)
        print(json.dumps(r), flush=True)
    x = qkv.clone().requires_grad_(True)
    o = ops.attention(x, plan, Hq, Hkv, D)
    g = torch.randn_like(o)
    t = timeit(lambda: torch.autograd.grad(ops.attention(x, plan, Hq, Hkv, D), x, g))
    r = {"kernel": "tree_attn_fwd_bwd", "T": T, "ms": t, "tflops": 3.5 * fl / t / 1e9}
    res.append(r)
    print(json.dumps(r), flush=True)
    # logprob head
    M, Hd, V = 4096, 3584, 152064
    h = torch.randn(M, Hd, device=dev).bfloat16()
    W = (torch.randn(V, Hd, device=dev) * 0.02).bfloat16()
    lab = torch.randint(0, V, (M,), device=dev, dtype=torch.int32)
    t = timeit(lambda: ops.ext().head_fwd(h, W, lab, 1.0, 0))
    fl = 2.0 * M * V * Hd
    r = {"kernel": "head_fwd", "M": M, "V": V, "ms": t, "tflops": fl / t / 1e9}
    res.append(r)
    print(json.dumps(r), flush=True)
    # decode attention: 256 requests x 3000 keys
    B, L = 256, 3000
    kc = torch.randn(B * L, Hkv * D, device=dev).bfloat16()
    vc = torch.randn(B * L, Hkv * D, device=dev).bfloat16()
    ip = torch.arange(0, B + 1, device=dev, dtype=torch.int32) * L
    idx = torch.randperm(B * L, device=dev).to(torch.int32)
    q = torch.randn(B, Hq * D, device=dev).bfloat16()
    by = 2.0 * B * L * Hkv * D * 2
    for persistent in (False, True):
        for splits in (4, 8):
            da = ops.DecodeAttention(Hq, Hkv, D, B, splits, dev, persistent=persistent)
            t = timeit(lambda: da(q, kc, vc, ip, idx))
            r = {"kernel": "decode_attn_persistent" if persistent else "decode_attn_splitk", "splits": splits,
                 "B": B, "L": L, "ms": t, "gbs": by / t / 1e6, "frac_of_measured": by / t / 1e6 / pk["hbm_gbs"]}
            res.append(r)
            print(json.dumps(r), flush=True)
    # shared-prefix case: 8 requests per group share a 2048-slot prefix (mounted task prefix)
    groups = B // 8
    pre = torch.randperm(B * L, device=dev)[: groups * 2048].view(groups, 2048).to(torch.int32)
    own = torch.randperm(B * L, device=dev)[: B * (L - 2048)].view(B, L - 2048).to(torch.int32)
    idx2 = torch.cat([pre.repeat_interleave(8, 0), own], 1).reshape(-1).contiguous()
    uniq = (groups * 2048 + B * (L - 2048)) * Hkv * D * 2 * 2
    for persistent in (False, True):
        da = ops.DecodeAttention(Hq, Hkv, D, B, 8, dev, persistent=persistent)
        t = timeit(lambda: da(q, kc, vc, ip, idx2))
        r = {"kernel": ("decode_attn_persistent" if persistent else "decode_attn_splitk") + "_shared_prefix",
             "B": B, "L": L, "ms": t, "logical_gbs": by / t / 1e6, "unique_gbs": uniq / t / 1e6}
        res.append(r)
        print(json.dumps(r), flush=True)
    ops.check_status(0)
    if args.json:
        with open(args.json, "w") as f:
            json.dump(res, f, indent=1)


if __name__ == "__main__":
    main()
