"""Run one kernel case a few times on a small input (for ncu captures and quick timing).

    python -m octopus_b200.tools.kernel_cases <case> [--reps N]

Cases (inputs sized above L2 where DRAM behaviour matters, a few GB at most):
  gemm_fwd_7b        X[16384, 3584] @ W[18944*2, 3584]^T (gate/up projection)
  gemm_wgrad_7b      dY^T X for the down projection (MN-major operands)
  attn_fwd_pp        tree attention forward, tcgen05 kernel with two query tiles per CTA
                     (8 x 2048 own + 2048 prefix)
  attn_fwd_mma       same on the mma.sync kernel (the path of head dims other than 128)
  attn_bwd           tree attention backward (dq + dkv kernels)
  decode_splitk      paged decode, 256 requests x 3000 keys (split-K kernel)
  decode_persistent  same on the persistent producer/consumer kernel
  decode_dag         persistent decode with the DAG solver stage's sharing: 32 instances x
                     8 rows; each row = shared 2048-token prefix + planner segment (shared
                     by 2 rows) + own 272 tokens
  decode_dag_flat    same lengths, every row's keys distinct (no sharing)
  decode_dag_shared  the decode_dag rows on the shared-prefix kernel (segments planned once)
  decode_gemms       the four GEMMs of one 7B decoder layer at 256 decode rows (OCTO_SPLITK=0: no split-K,
                     OCTO_GEMM_MT=1: one M-tile per CTA)
  decode_gemm_{qkv,o,gu,down}  one of them, over weight copies > 2x L2 (time / copies = per GEMM)
  decode_sweep       the four decode GEMMs at 16..256 rows: time, HBM rate, roofline fraction
  head_fwd           fused logprob head, 4096 rows x 152064 vocab
  sample_head        fused sampling head, 256 rows x 152064 vocab
"""
from __future__ import annotations

import argparse
import time

import numpy as np
import torch

from octopus_b200 import ops


def tree_case(dev):
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
    return plan, qkv, Hq, Hkv, D


def decode_case(dev):
    B, L, Hq, Hkv, D = 256, 3000, 28, 4, 128
    kc = torch.randn(B * L, Hkv * D, device=dev).bfloat16()
    vc = torch.randn(B * L, Hkv * D, device=dev).bfloat16()
    ip = torch.arange(0, B + 1, device=dev, dtype=torch.int32) * L
    idx = torch.randperm(B * L, device=dev).to(torch.int32)
    q = torch.randn(B, Hq * D, device=dev).bfloat16()
    return q, kc, vc, ip, idx, Hq, Hkv, D, B


def decode_dag_rows(share: bool):
    n_inst, per, pre, plan, own = 32, 8, 2048, 528, 272
    rows, ctx, nxt = [], [], 0

    def take(n):
        nonlocal nxt
        r = np.arange(nxt, nxt + n)
        nxt += n
        return r

    for i in range(n_inst):
        p = take(pre)
        for s in range(per // 2):
            pl = take(plan)
            for k in range(2):
                rows.append(np.concatenate([p, pl, take(own)]) if share else take(pre + plan + own))
                ctx.append(pre + plan)
    return rows, np.asarray(ctx), nxt


def decode_dag_case(dev, share: bool):
    Hq, Hkv, D = 28, 4, 128
    n_inst, per, pre, plan, own = 32, 8, 2048, 528, 272
    B = n_inst * per
    rows, nxt = [], 0

    def take(n):
        nonlocal nxt
        r = np.arange(nxt, nxt + n)
        nxt += n
        return r

    for i in range(n_inst):
        p = take(pre)
        for s in range(per // 2):
            pl = take(plan)
            for k in range(2):
                if share:
                    rows.append(np.concatenate([p, pl, take(own)]))
                else:
                    rows.append(take(pre + plan + own))
    L = len(rows[0])
    idx = torch.from_numpy(np.concatenate(rows).astype(np.int32)).to(dev)
    kc = torch.randn(nxt, Hkv * D, device=dev).bfloat16()
    vc = torch.randn(nxt, Hkv * D, device=dev).bfloat16()
    ip = torch.arange(0, B + 1, device=dev, dtype=torch.int32) * L
    q = torch.randn(B, Hq * D, device=dev).bfloat16()
    return q, kc, vc, ip, idx, Hq, Hkv, D, B


def build(case: str, dev):
    if case == "gemm_fwd_7b":
        A = torch.randn(16384, 3584, device=dev).bfloat16()
        W = torch.randn(2 * 18944, 3584, device=dev).bfloat16()
        C = torch.empty(16384, 2 * 18944, device=dev, dtype=torch.bfloat16)
        return lambda: ops.gemm(A, W, out=C)
    if case == "gemm_wgrad_7b":
        dY = torch.randn(16384, 3584, device=dev).bfloat16()
        X = torch.randn(16384, 18944, device=dev).bfloat16()
        G = torch.zeros(3584, 18944, device=dev)
        return lambda: ops.gemm(dY, X, a_mn=True, b_mn=True, out=G, accumulate=True)
    if case in ("attn_fwd_pp", "attn_fwd_mma"):
        plan, qkv, Hq, Hkv, D = tree_case(dev)
        q, k, v = qkv[:, : Hq * D], qkv[:, Hq * D: (Hq + Hkv) * D], qkv[:, (Hq + Hkv) * D:]
        mode = {"attn_fwd_pp": 2, "attn_fwd_mma": 0}[case]
        return lambda: ops.ext().attn_fwd(q, k, v, plan.cu_q, plan.cu_k, plan.key_idx, plan.tiles_for(mode), Hq, Hkv,
                                          D, D ** -0.5, True, True, mode)
    if case == "attn_bwd":
        plan, qkv, Hq, Hkv, D = tree_case(dev)
        x = qkv.clone().requires_grad_(True)
        o = ops.attention(x, plan, Hq, Hkv, D)
        g = torch.randn_like(o)
        return lambda: torch.autograd.grad(o, x, g, retain_graph=True)
    if case in ("decode_splitk", "decode_persistent"):
        q, kc, vc, ip, idx, Hq, Hkv, D, B = decode_case(dev)
        da = ops.DecodeAttention(Hq, Hkv, D, B, 8, dev, persistent=case == "decode_persistent")
        return lambda: da(q, kc, vc, ip, idx)
    if case == "decode_gemms":
        M, H, F = 256, 3584, 18944
        x = torch.randn(M, H, device=dev).bfloat16()
        ws = [(torch.randn(n, k, device=dev) * 0.02).bfloat16() for n, k in ((4608, H), (H, 3584), (2 * F, H), (H, F))]
        xa = torch.randn(M, 3584, device=dev).bfloat16()
        xf = torch.randn(M, F, device=dev).bfloat16()
        ins = (x, xa, x, xf)
        return lambda: [ops.gemm(i, w) for i, w in zip(ins, ws)]
    if case.startswith("decode_gemm_"):
        # one decode GEMM, rotating over weight copies that together exceed 2x L2 (cold weights)
        M, H, F = 256, 3584, 18944
        n, k = {"qkv": (4608, H), "o": (H, 3584), "gu": (2 * F, H), "down": (H, F)}[case[len("decode_gemm_"):]]
        copies = max(1, -(-(300 << 20) // (n * k * 2)))
        ws = [(torch.randn(n, k, device=dev) * 0.02).bfloat16() for _ in range(copies)]
        x = torch.randn(M, k, device=dev).bfloat16()
        return lambda: [ops.gemm(x, w) for w in ws]
    if case == "decode_dag_shared":
        Hq, Hkv, D = 28, 4, 128
        rows, ctx, nslots = decode_dag_rows(True)
        B = len(rows)
        kc = torch.randn(nslots, Hkv * D, device=dev).bfloat16()
        vc = torch.randn(nslots, Hkv * D, device=dev).bfloat16()
        starts = np.cumsum([0] + [len(r) for r in rows[:-1]]).astype(np.int32)
        idx = torch.from_numpy(np.concatenate(rows).astype(np.int32)).to(dev)
        ln = torch.tensor([len(r) for r in rows], dtype=torch.int32, device=dev)
        q = torch.randn(B, Hq * D, device=dev).bfloat16()
        sd = ops.SharedDecode(Hq, Hkv, D, B, dev)
        assert sd.plan(rows, starts, ctx, np.asarray([len(r) for r in rows]), B)
        return lambda: sd(q, kc, vc, idx, ln)
    if case in ("decode_dag", "decode_dag_flat"):
        q, kc, vc, ip, idx, Hq, Hkv, D, B = decode_dag_case(dev, case == "decode_dag")
        da = ops.DecodeAttention(Hq, Hkv, D, B, 8, dev, persistent=True)
        return lambda: da(q, kc, vc, ip, idx)
    if case in ("head_fwd", "sample_head"):
        M = 4096 if case == "head_fwd" else 256
        h = torch.randn(M, 3584, device=dev).bfloat16()
        W = (torch.randn(152064, 3584, device=dev) * 0.02).bfloat16()
        lab = torch.randint(0, 152064, (M,), device=dev, dtype=torch.int32)
        if case == "head_fwd":
            return lambda: ops.ext().head_fwd(h, W, lab, 1.0, 0)
        st = torch.arange(M, device=dev, dtype=torch.int64)
        return lambda: ops.ext().sample_head(h, W, 1.0, 1, st, 0)
    raise SystemExit(f"unknown case {case}")


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("case")
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--graph", action="store_true", help="time CUDA-graph replays (no host launch overhead)")
    args = ap.parse_args(argv)
    dev = torch.device("cuda", 0)
    fn = build(args.case, dev)
    fn()
    torch.cuda.synchronize()
    run = fn
    if args.graph:
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            fn()
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        run = g.replay
        run()
        torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.reps):
        run()
    b.record()
    torch.cuda.synchronize()
    ops.check_status(0)
    print(f"{args.case}: {a.elapsed_time(b) / args.reps:.3f} ms/iter")


def decode_sweep(rows=(16, 32, 64, 128, 256), reps=20):
    """The four decode GEMMs of a 7B layer at several decode batch sizes: CUDA-graph replays over
    weight copies that together exceed 2x L2 (cold weights), per-GEMM time, achieved HBM bandwidth
    and the fraction of the roofline max(weight bytes / HBM copy rate, FLOPs / bf16 GEMM rate)
    (MEASURED_PEAKS.json when present, else 6.65 TB/s and 1.59 PFLOP/s)."""
    import json
    import os

    dev = torch.device("cuda", 0)
    hbm, tflops = 6650.0, 1590.0
    peaks = os.path.join(os.path.dirname(__file__), "..", "..", "MEASURED_PEAKS.json")
    if os.path.exists(peaks):
        with open(peaks) as f:
            pk = json.load(f)
        hbm, tflops = float(pk.get("hbm_gbs", hbm)), float(pk.get("bf16_tflops", tflops))
    H, F = 3584, 18944
    shapes = {"qkv": (4608, H), "o": (H, 3584), "gu": (2 * F, H), "down": (H, F)}
    for name, (n, k) in shapes.items():
        copies = max(2, -(-(300 << 20) // (n * k * 2)))
        ws = [(torch.randn(n, k, device=dev) * 0.02).bfloat16() for _ in range(copies)]
        for M in rows:
            x = torch.randn(M, k, device=dev).bfloat16()
            outs = [torch.empty(M, n, device=dev, dtype=torch.bfloat16) for _ in ws]

            def fn():
                for w, o in zip(ws, outs):
                    ops.gemm(x, w, out=o)

            fn()
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                fn()
            torch.cuda.current_stream().wait_stream(s)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                fn()
            for _ in range(3):
                g.replay()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            a.record()
            for _ in range(reps):
                g.replay()
            b.record()
            torch.cuda.synchronize()
            ops.check_status(0)
            us = a.elapsed_time(b) * 1e3 / (reps * copies)
            byts = n * k * 2 + M * (n + k) * 2
            roof = max(byts / (hbm * 1e3), 2.0 * M * n * k / (tflops * 1e6))  # microseconds
            print(json.dumps({"gemm": name, "M": M, "N": n, "K": k, "us": round(us, 2),
                              "tb_s": round(byts / us / 1e6, 2), "roofline_us": round(roof, 2),
                              "frac_of_roofline": round(roof / us, 3)}), flush=True)
            del g
        del ws


def trace_attn_tc():
    """Per-event timeline (microseconds from CTA start) of CTA (0, 0) of the tcgen05 attention."""
    dev = torch.device("cuda", 0)
    plan, qkv, Hq, Hkv, D = tree_case(dev)
    q, k, v = qkv[:, : Hq * D], qkv[:, Hq * D: (Hq + Hkv) * D], qkv[:, (Hq + Hkv) * D:]
    tr = torch.zeros(10 * 64, dtype=torch.int64, device=dev)
    for _ in range(2):
        ops.ext().attn_fwd(q, k, v, plan.cu_q, plan.cu_k, plan.key_idx, plan.fwd_tiles, Hq, Hkv, D, D ** -0.5, True,
                           True, 1, tr)
    torch.cuda.synchronize()
    t = tr.view(10, 64).cpu().numpy().astype(np.int64)
    t0 = t[9, 0]
    names = ["prod_empty_ok", "prod_issued", "mma_kv_full", "mma_S_issued", "mma_p_full", "sm_s_full",
             "sm_s_loaded", "sm_o_done", "sm_p_stored"]
    n = int((t[3] > 0).sum())
    print("CTA total us", (t[9, 1] - t0) / 1e3, "tiles", n)
    for j in range(min(n, 12)):
        print(j, " ".join(f"{nm}={(t[r, j] - t0) / 1e3:.2f}" for r, nm in enumerate(names) if t[r, j] > 0))


if __name__ == "__main__":
    import sys
    if len(sys.argv) > 1 and sys.argv[1] == "trace_attn_tc":
        trace_attn_tc()
    elif len(sys.argv) > 1 and sys.argv[1] == "decode_sweep":
        decode_sweep()
    else:
        main()
