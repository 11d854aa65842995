"""Fused compute + collective kernels against their NCCL baselines, on N GPUs.

    torchrun --nproc-per-node N -m octopus_b200.tools.bench_comm [--json out.json]

One rank per GPU.  Each case is timed with CUDA events on every rank after warm-up
(median of repeats, a barrier before each repeat) and reported as the MAX over ranks.
For every fused kernel the same op is also timed on the baseline path (NCCL collective +
the same GEMM or optimizer kernel), and the roofline time is the slower of its FLOPs at
the measured bf16 peak and the bytes each GPU must move over NVLink at the measured peer
bandwidth (770 GB/s per direction).  Cases (7B shapes):

  ag_gemm   x [N * rows_s, 3584] all-gathered (sequence-sharded) -> x @ W^T for the
            column-parallel qkv (W [4608 / N, 3584]) and gate/up (W [37888 / N, 3584])
            projections; baseline: all_gather_into_tensor + GEMM
  gemm_rs   a [N * rows_s, K / N] @ W^T -> reduce-scatter of [N * rows_s, 3584] plus the
            residual add and the next RMSNorm (tp_reduce) for the o (K 3584) and down (K
            18944) projections; baseline: GEMM + reduce_scatter_tensor + add + RMSNorm
  rs_sum_sq sharded gradient reduce-scatter + squared norm over a 2 GiB fp32 gradient;
            baseline: reduce_scatter_tensor + norm
  adamw_bcast  AdamW on the owned shard + peer stores of the new bf16 weights to every rank;
            baseline: AdamW + all_gather_into_tensor
  fsdp_layer_gather / fsdp_layer_reduce_scatter  the full-shard actor's per-layer all-gather of
            one 7B decoder layer's bf16 shards and reduce-scatter-accumulate of its fp32
            gradient; baseline: all_gather_into_tensor / reduce_scatter_tensor + add
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
from datetime import timedelta

import torch
import torch.distributed as dist

LINK_GBS = 770.0  # measured peer copy, GB/s per direction per GPU


def _peaks():
    p = os.path.join(os.path.dirname(__file__), "..", "..", "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return json.load(f)
    except OSError:
        return {"bf16_tflops": 1590.0, "hbm_gbs": 6650.0}


def timed(fn, reps: int = 20, warmup: int = 5) -> float:
    """Median ms of fn on this rank, max over ranks (barrier before every repeat)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(reps):
        dist.barrier()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b))
    t = torch.tensor([statistics.median(ts)], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t)


def roofline_ms(flops: float, link_bytes: float, pk: dict) -> float:
    return max(flops / (pk["bf16_tflops"] * 1e12), link_bytes / (LINK_GBS * 1e9)) * 1e3


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--json", default=None)
    ap.add_argument("--reps", type=int, default=20)
    args = ap.parse_args(argv)
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    from octopus_b200 import ops
    from octopus_b200.parallel.peer import PeerBuffers
    from octopus_b200.parallel.tp import TPGroup

    rank, world = dist.get_rank(), dist.get_world_size()
    pk = _peaks()
    H, F, QKV = 3584, 18944, 4608
    rows_list = (64, 128, 2048)
    comm = TPGroup(dist.group.WORLD, dev, max_rows=world * max(rows_list), hidden=H, max_n=H, max_sample_rows=256)
    out = []

    def emit(rec):
        out.append(rec)
        if rank == 0:
            print(json.dumps(rec), flush=True)

    torch.manual_seed(0)
    for name, n_full in (("qkv", QKV), ("gate_up", 2 * F)):
        W = (torch.randn(n_full // world, H, device=dev) * 0.02).bfloat16()
        for rows_s in rows_list:
            M = world * rows_s
            x = comm.x_local(rows_s)
            x.copy_((torch.randn(rows_s, H, device=dev)).bfloat16())
            y = torch.empty(M, n_full // world, dtype=torch.bfloat16, device=dev)
            xg = torch.empty(M, H, dtype=torch.bfloat16, device=dev)
            xl = x.clone()

            def fused():
                comm.ag_linear(rows_s, W, y)

            def base():
                dist.all_gather_into_tensor(xg, xl)
                ops.gemm(xg, W, out=y)

            tf, tb = timed(fused, args.reps), timed(base, args.reps)
            flops = 2.0 * M * (n_full // world) * H
            link = (world - 1) * rows_s * H * 2.0
            roof = roofline_ms(flops, link, pk)
            emit({"kernel": "ag_gemm", "proj": name, "world": world, "rows_per_rank": rows_s, "M": M,
                  "N": n_full // world, "K": H, "fused_ms": round(tf, 4), "nccl_ms": round(tb, 4),
                  "link_bytes": link, "link_gbs": round(link / tf / 1e6, 1), "tflops": round(flops / tf / 1e9, 1),
                  "roofline_ms": round(roof, 4), "frac_of_roofline": round(roof / tf, 3),
                  "speedup_vs_nccl": round(tb / tf, 2)})
    for name, k_full in (("o", H), ("down", F)):
        W = (torch.randn(H, k_full // world, device=dev) * 0.02).bfloat16()
        wn = torch.ones(H, dtype=torch.bfloat16, device=dev)
        for rows_s in rows_list:
            M = world * rows_s
            A = (torch.randn(M, k_full // world, device=dev) * 0.5).bfloat16()
            h = torch.zeros(rows_s, H, dtype=torch.bfloat16, device=dev)
            x = comm.x_local(rows_s)
            part = torch.empty(M, H, dtype=torch.bfloat16, device=dev)
            shard = torch.empty(rows_s, H, dtype=torch.bfloat16, device=dev)

            def fused():
                g = comm.rs_linear(A, W)
                comm.reduce(h, g, w=wn, x=x, eps=1e-6)

            def base():
                ops.gemm(A, W, out=part)
                dist.reduce_scatter_tensor(shard, part)
                h.add_(shard)
                ops.rmsnorm(h, wn, 1e-6)

            tf, tb = timed(fused, args.reps), timed(base, args.reps)
            flops = 2.0 * M * H * (k_full // world)
            link = (world - 1) * rows_s * H * 2.0
            roof = roofline_ms(flops, link, pk)
            emit({"kernel": "gemm_rs", "proj": name, "world": world, "rows_per_rank": rows_s, "M": M, "N": H,
                  "K": k_full // world, "fused_ms": round(tf, 4), "nccl_ms": round(tb, 4), "link_bytes": link,
                  "link_gbs": round(link / tf / 1e6, 1), "tflops": round(flops / tf / 1e9, 1),
                  "roofline_ms": round(roof, 4), "frac_of_roofline": round(roof / tf, 3),
                  "speedup_vs_nccl": round(tb / tf, 2)})
    comm.close()
    # ------------------------------------------------------------------ actor collectives
    C = ops.ext()
    total = (1 << 29) // world * world  # 512 Mi fp32 gradient elements (2 GiB)
    shard = total // world
    grads = PeerBuffers(total * 4, dev)
    weights = PeerBuffers(total * 2, dev)
    g = grads.local.view(torch.float32)
    g.normal_()
    w16 = weights.local.view(torch.bfloat16)
    master = torch.randn(shard, device=dev)
    m1, m2 = torch.zeros_like(master), torch.zeros_like(master)
    gs = torch.zeros_like(master)
    sq = torch.zeros(1, device=dev)
    off = rank * shard
    sh16 = torch.empty(shard, dtype=torch.bfloat16, device=dev)

    def rs_fused():
        sq.zero_()
        C.rs_sum_sq(grads.ptrs, off, gs, sq)

    def rs_base():
        dist.reduce_scatter_tensor(gs, g)
        sq.zero_()
        ops.sqnorm_(gs, sq)

    tf, tb = timed(rs_fused, 10, 2), timed(rs_base, 10, 2)
    link = (world - 1) * shard * 4.0  # bytes each rank reads from its peers
    roof = roofline_ms(0.0, link, pk)
    emit({"kernel": "rs_sum_sq", "world": world, "elements": total, "fused_ms": round(tf, 3), "nccl_ms": round(tb, 3),
          "link_bytes": link, "link_gbs": round(link / tf / 1e6, 1), "roofline_ms": round(roof, 3),
          "frac_of_roofline": round(roof / tf, 3), "speedup_vs_nccl": round(tb / tf, 2)})

    def adam_fused():
        C.adamw_bcast(master, gs, m1, m2, weights.ptrs, off, 1e-6, 0.9, 0.999, 1e-8, 0.0, 1, sq, 1.0, 1.0)

    def adam_base():
        ops.adamw_(master, gs, m1, m2, sh16, lr=1e-6, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.0, step=1,
                   sqnorm=sq, max_norm=1.0)
        dist.all_gather_into_tensor(w16, sh16)

    tf, tb = timed(adam_fused, 10, 2), timed(adam_base, 10, 2)
    link = (world - 1) * shard * 2.0  # bytes each rank stores to its peers
    roof = roofline_ms(0.0, link, pk)
    emit({"kernel": "adamw_bcast", "world": world, "elements": total, "fused_ms": round(tf, 3),
          "nccl_ms": round(tb, 3), "link_bytes": link, "link_gbs": round(link / tf / 1e6, 1),
          "roofline_ms": round(roof, 3), "frac_of_roofline": round(roof / tf, 3), "speedup_vs_nccl": round(tb / tf, 2)})
    # ------------------------------------------------------------------ full-shard actor: one 7B layer unit
    unit = 233_046_016 // (world * 8) * (world * 8)  # elements of one decoder layer unit (padded to world * 8)
    su = unit // world
    shards = PeerBuffers(su * 2, dev)
    shards.local.view(torch.bfloat16).normal_()
    slot = torch.empty(unit, dtype=torch.bfloat16, device=dev)
    gslots = PeerBuffers(unit * 4, dev)
    gsl = gslots.local.view(torch.float32)
    gsl.normal_()
    acc = torch.zeros(su, device=dev)
    mine = shards.local.view(torch.bfloat16)[:su]

    def ag_fused():
        C.peer_gather_bf16(shards.ptrs, 0, su, slot)

    def ag_base():
        dist.all_gather_into_tensor(slot, mine)

    tf, tb = timed(ag_fused, 10, 2), timed(ag_base, 10, 2)
    link = (world - 1) * su * 2.0
    roof = roofline_ms(0.0, link, pk)
    emit({"kernel": "fsdp_layer_gather", "world": world, "elements": unit, "fused_ms": round(tf, 3),
          "nccl_ms": round(tb, 3), "link_bytes": link, "link_gbs": round(link / tf / 1e6, 1),
          "roofline_ms": round(roof, 3), "frac_of_roofline": round(roof / tf, 3), "speedup_vs_nccl": round(tb / tf, 2)})
    red = torch.empty(su, device=dev)

    def rsl_fused():
        C.peer_rs_acc(gslots.ptrs, rank * su, acc)

    def rsl_base():
        dist.reduce_scatter_tensor(red, gsl)
        acc.add_(red)

    tf, tb = timed(rsl_fused, 10, 2), timed(rsl_base, 10, 2)
    link = (world - 1) * su * 4.0
    roof = roofline_ms(0.0, link, pk)
    emit({"kernel": "fsdp_layer_reduce_scatter", "world": world, "elements": unit, "fused_ms": round(tf, 3),
          "nccl_ms": round(tb, 3), "link_bytes": link, "link_gbs": round(link / tf / 1e6, 1),
          "roofline_ms": round(roof, 3), "frac_of_roofline": round(roof / tf, 3), "speedup_vs_nccl": round(tb / tf, 2)})
    torch.cuda.synchronize()
    dist.barrier()
    shards.close()
    gslots.close()
    grads.close()
    weights.close()
    ops.check_status(local)
    if rank == 0 and args.json:
        with open(args.json, "w") as f:
            json.dump(out, f, indent=1)
    dist.barrier()
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
