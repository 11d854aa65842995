#!/usr/bin/env python
"""Headline benchmark: RL step tokens/sec/box (rollout + prefix-tree train + weight sync)
on the Qwen2.5-7B-shape multi-agent DAG config (planner -> 2 solvers -> verifier, shared
2048-token prefix mounted zero-copy into every agent, 512-token turns, 32 DAG
instances x 4 samples), bf16, synthetic tokens, random-init weights.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl octopus|reference]

N > 1 is launched by torchrun (one rank per GPU).  Scaling is strong: the whole config
(32 x 4 DAG samples) is split across N / tp rollout replicas, each a tensor-parallel
group of `--tp` GPUs (default 2, the config's TP=2) running the fused AG->GEMM /
GEMM->RS engine; the actor is ZeRO-sharded over all N ranks (fused peer-memory
reduce-scatter + AdamW + all-gather), and the ranks of a TP group split the training of
their group's rollout.  `value` = generated tokens of all replicas per second of device
time (CUDA events on each rank, max over ranks), every generated token is also trained
once.  `e2e` = the same metric from the per-step wall clock of the
public `RLTrainer.step()` API, whose timed region includes the host->device copies of
each step's inputs (prompts, tree plans) from pinned memory and the device->host reads
of the results (sampled tokens, logprobs, loss).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "RL step tokens/sec/box (rollout+train+sync), 7B-shape multi-agent, 1/2/4/8 B200"
METRIC_GRPO = "RL step tokens/sec/box (rollout+train+sync), 1.5B-shape single-agent GRPO"
BASELINE_VALUE = None  # the reference publishes no tokens/sec figure for this metric


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="octopus", choices=["octopus", "reference"])
    ap.add_argument("--config", default="dag7b", choices=["dag7b", "grpo1.5b"],
                    help="dag7b: BASELINE config 3 (the headline); grpo1.5b: config 2 (1.5B single-agent GRPO, "
                         "64 prompts x 8 samples x 1024 tokens, TP=1 replicas)")
    ap.add_argument("--model", default="")
    ap.add_argument("--instances", type=int, default=32)
    ap.add_argument("--samples", type=int, default=4)
    ap.add_argument("--prefix", type=int, default=2048)
    ap.add_argument("--turn", type=int, default=512)
    ap.add_argument("--role", type=int, default=16)
    ap.add_argument("--mb-tokens", type=int, default=32768)
    ap.add_argument("--kv-gb", type=float, default=0.0, help="KV pool size (0: sized from the config)")
    ap.add_argument("--layers", type=int, default=0, help="override layer count (smoke tests only)")
    ap.add_argument("--no-graphs", action="store_true")
    ap.add_argument("--tp", type=int, default=0, help="rollout tensor parallelism (0: 2 when N is even, else 1)")
    ap.add_argument("--mode", default="colocated", choices=["colocated", "disagg"],
                    help="N > 1: colocated (every GPU rolls out, then trains) or disagg (half of the GPUs roll out "
                         "while the other half trains on the previous rollout, rl.disagg)")
    ap.add_argument("--rollout-gpus", type=int, default=0, help="--mode disagg: rollout GPUs (0: half, rounded up)")
    ap.add_argument("--profile-step", default="",
                    help="after the timed steps, run one more step under the PyTorch CUDA trace and write rank 0's "
                         "per-kernel breakdown (JSON) here; not part of the timed value")
    ap.add_argument("--fsdp-gather", action="store_true",
                    help="--actor fsdp: gather each layer's weights from the shards (default: read the serving copy)")
    ap.add_argument("--actor", default="sharded", choices=["sharded", "fsdp", "dp"],
                    help="N > 1 actor: sharded (ZeRO: fp32 master / optimizer sharded, fused peer-memory RS + AdamW + "
                         "all-gather), fsdp (full shard: per-layer peer-memory gather and reduce-scatter), or dp "
                         "(replicated + NCCL all-reduce)")
    return ap.parse_args()


def reference_arm(args):
    reason = ("reference stack not installable offline: its build backend (hatchling) is not in the wheelhouse, and "
              "its RL step needs sglang 0.5.19, AReaL and peft, none of which is installed")
    print(json.dumps({"impl": "reference", "metric": METRIC, "unavailable": reason, "n_gpus": args.gpus}))
    return 0


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.p = None

    def start(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.QUERY}",
                                       "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.f,
                                      stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

    def stop(self) -> dict:
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.p.kill()
        self.f.flush()
        self.f.seek(0)
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.f.read().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        os.unlink(self.f.name)
        load = [x for x in sm if smax and x > 0.3 * smax] or sm
        return {"sm_mhz": statistics.median(load) if load else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


def main():
    args = parse()
    if args.impl == "reference":
        return reference_arm(args)
    os.environ.setdefault("PYTORCH_CUDA_ALLOC_CONF", "expandable_segments:True")
    import torch
    import torch.distributed as dist

    from octopus_b200 import ops
    from octopus_b200.envs.dag import DagConfig, MultiAgentDag
    from octopus_b200.models.config import get_config
    from octopus_b200.parallel.dp import DataParallel
    from octopus_b200.parallel.fsdp import ShardedActor
    from octopus_b200.rl.actor import Actor
    from octopus_b200.rl.trainer import RLTrainer, TrainerConfig
    from octopus_b200.serving.engine import Engine
    from octopus_b200.serving.tp_engine import TPEngine
    from octopus_b200.utils import iostats

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=dev)
    n_gpus = world

    if world > 1 and args.mode == "disagg":
        return run_disagg(args, world, rank, local, dev)
    over = {"layers": args.layers} if args.layers else {}
    grpo = args.config == "grpo1.5b"
    args.model = args.model or ("qwen2.5-1.5b" if grpo else "qwen2.5-7b")
    cfg = get_config(args.model, **over)
    tp = 1 if grpo else (args.tp or (2 if world % 2 == 0 else 1))
    if world % tp:
        raise SystemExit(f"--tp {tp} must divide the {world} GPUs")
    replicas = world // tp
    rep, tp_rank = rank // tp, rank % tp
    tp_group = None
    if tp > 1:
        for r in range(replicas):  # every rank creates every group, in the same order
            g = dist.new_group(list(range(r * tp, (r + 1) * tp)))
            if r == rep:
                tp_group = g
    # strong scaling: this replica's share of the DAG instances (or GRPO prompts)
    if grpo:
        from octopus_b200.envs.grpo import GrpoConfig, SingleAgentGrpo

        gcfg = GrpoConfig(seed=1000 + rep)
        inst = [i for i in range(gcfg.prompts) if i % replicas == rep]
        env = SingleAgentGrpo(cfg.vocab_size, gcfg)
    else:
        inst = [i for i in range(args.instances) if i % replicas == rep]
        dcfg = DagConfig(instances=args.instances, samples=args.samples, prefix_len=args.prefix, turn_len=args.turn,
                         role_len=args.role, seed=1000 + rep)
        env = MultiAgentDag(cfg.vocab_size, dcfg)
    sharded = world > 1 and args.actor in ("sharded", "fsdp")
    if world > 1 and args.actor == "fsdp":
        from octopus_b200.parallel.fsdp import FSDPActor

        actor = FSDPActor(cfg, dev, seed=0, gather_weights=args.fsdp_gather)
    else:
        actor = ShardedActor(cfg, dev, seed=0) if sharded else Actor(cfg, dev, seed=0)
    if grpo:
        per_inst = gcfg.prompt_len + gcfg.samples * (gcfg.response_len + 1)
    else:
        per_inst = args.prefix + args.samples * (4 * (args.turn + args.role) + 2)
    kv_slots = int(len(inst) * per_inst * 1.15) + 8192
    if args.kv_gb:
        kv_slots = int(args.kv_gb * (1 << 30) / (4 * cfg.layers * cfg.kv_width // tp))
    rows = len(inst) * (gcfg.samples if grpo else args.samples * 2)
    max_batch = max(8 * tp, 1 << (rows - 1).bit_length())
    if tp > 1:
        engine = TPEngine(cfg, actor.weights, group=tp_group, kv_slots=kv_slots, max_batch=max_batch, device=dev,
                          use_graphs=not args.no_graphs)
    else:
        engine = Engine(cfg, actor.weights, kv_slots=kv_slots, max_batch=max_batch, device=dev,
                        use_graphs=not args.no_graphs)
    dp = DataParallel(actor) if world > 1 and not sharded else None

    class _Env:
        def rollout(self, eng):
            return env.rollout(eng, inst)

    trainer = RLTrainer(actor, engine, _Env(), TrainerConfig(mb_tokens=args.mb_tokens, mb_shard=(tp_rank, tp)),
                        sync_fn=engine.sync_weights if tp > 1 else None)
    if dp is not None:
        dp.attach(trainer)

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        trainer.step()
    torch.cuda.synchronize()
    ops.check_status(local)
    barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    e0 = dict(engine.stats)
    clocks.start()
    iostats.reset()
    l0 = ops.launches()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    gen, wall, stats = 0, [], []
    start.record()
    for _ in range(args.steps):
        t0 = time.perf_counter()
        st = trainer.step()
        torch.cuda.synchronize()
        wall.append(time.perf_counter() - t0)
        gen += st["generated_tokens"] if tp_rank == 0 else 0  # a TP group's rollout counted once
        stats.append(st)
    end.record()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    clk = clocks.stop()
    io = iostats.snapshot()
    launches = ops.launches() - l0
    ms = start.elapsed_time(end)
    ops.check_status(local)
    t = torch.tensor([ms, float(gen), float(launches), io["h2d"], io["d2h"], sum(wall)], dtype=torch.float64,
                     device=dev)
    if world > 1:
        mx = t.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        sm = t.clone()
        dist.all_reduce(sm, op=dist.ReduceOp.SUM)
        ms, wall_s = float(mx[0]), float(mx[5])
        gen, launches, h2d_b, d2h_b = float(sm[1]), int(sm[2]), float(sm[3]), float(sm[4])
    else:
        wall_s = sum(wall)
        h2d_b, d2h_b = float(io["h2d"]), float(io["d2h"])
    value = gen / (ms / 1000.0)
    e2e = gen / wall_s
    par = (f"rollout tp{tp} x {replicas} replicas" + (" (fused AG->GEMM / GEMM->RS)" if tp > 1 else "")
           + f", actor {dict(sharded='zero-sharded fused', fsdp='full-shard fused', dp='replicated')[args.actor]}"
           + f" over {n_gpus}"
           if n_gpus > 1 else "single GPU (rollout engine + actor colocated)")
    if grpo:
        metric = METRIC_GRPO
        run_config = {"model": args.model + (f"-L{args.layers}" if args.layers else ""), "config": "BASELINE config 2",
                      "global_batch": gcfg.prompts * gcfg.samples, "seq_len": gcfg.prompt_len + gcfg.response_len,
                      "parallelism": par, "prompts": gcfg.prompts, "samples": gcfg.samples,
                      "response_len": gcfg.response_len, "tokens_counted": "generated (= trained) tokens per RL step",
                      "l2": "inputs larger than L2 (KV > 10 GB per step)"}
    else:
        metric = METRIC
        run_config = {"model": args.model + (f"-L{args.layers}" if args.layers else ""),
                      "global_batch": args.instances * args.samples,
                      "seq_len": args.prefix + 4 * (args.turn + args.role), "parallelism": par,
                      "dag": "planner->2 solvers->verifier, prefix mounted zero-copy",
                      "instances": args.instances, "samples": args.samples, "prefix": args.prefix,
                      "turn": args.turn, "tokens_counted": "generated (= trained) tokens per RL step",
                      "l2": "inputs larger than L2 (7B weights 15 GB, KV > 10 GB per step)"}
    if rank == 0:
        s0 = stats[-1]
        out = {
            "metric": metric, "value": round(value, 2), "unit": "tokens/s", "n_gpus": n_gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 2), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None if BASELINE_VALUE is None else value / BASELINE_VALUE,
            "dtype": "bf16", "data": "synthetic (uniform random tokens, random-init weights, Bernoulli(0.5) rewards)",
            "config": run_config,
            "clocks": clk,
            "e2e": {"value": round(e2e, 2), "unit": "tokens/s", "h2d_bytes_per_step": int(h2d_b / args.steps),
                    "d2h_bytes_per_step": int(d2h_b / args.steps),
                    "api": "octopus_b200.rl.trainer.RLTrainer.step"},
            "gpu_launches": int(launches),
            "phases_s": {"rollout": round(s0["rollout_s"], 3), "train": round(s0["train_s"], 3),
                         "sync": round(s0["sync_s"], 4)},
            "engine_per_step": {k: round((engine.stats[k] - e0[k]) / args.steps, 3)
                                for k in ("prefill_s", "decode_s", "decode_steps", "prefill_tokens", "cached_tokens")},
            "tree_tokens": s0.get("tree_tokens"), "flat_tokens": s0.get("flat_tokens"),
        }
        print(json.dumps(out), flush=True)
    if args.profile_step:
        from torch.profiler import ProfilerActivity, profile

        from octopus_b200.tools.step_profile import breakdown

        if rank == 0:
            with profile(activities=[ProfilerActivity.CUDA]) as prof:
                st = trainer.step()
                torch.cuda.synchronize()
            out = breakdown(prof, st)
            with open(args.profile_step, "w") as f:
                json.dump(out, f, indent=1)
        else:
            trainer.step()
            torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        torch.cuda.synchronize()
        if tp > 1:
            engine._graphs.clear()
            engine.close()
        if sharded:
            actor.close()
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_disagg(args, world, rank, local, dev):
    """--mode disagg: ranks [0, R) roll out (one engine replica each, TP 1), ranks [R, N) train
    the previous iteration's rollouts (full-shard actor over the trainer ranks); rollouts and
    weights are exchanged between iterations (octopus_b200.rl.disagg)."""
    import torch
    import torch.distributed as dist

    from octopus_b200 import ops
    from octopus_b200.envs.dag import DagConfig, MultiAgentDag
    from octopus_b200.models.config import get_config
    from octopus_b200.rl.actor import Actor
    from octopus_b200.rl.disagg import DisaggRLTrainer, make_groups, rollout_weights, split_roles
    from octopus_b200.serving.engine import Engine
    from octopus_b200.utils import iostats

    if args.config != "dag7b":
        raise SystemExit("--mode disagg runs the dag7b config")
    over = {"layers": args.layers} if args.layers else {}
    args.model = args.model or "qwen2.5-7b"
    cfg = get_config(args.model, **over)
    n_roll = split_roles(world, args.rollout_gpus)
    n_train = world - n_roll
    train_group, push = make_groups(world, n_roll)
    role = "rollout" if rank < n_roll else "train"
    if role == "rollout":
        inst = [i for i in range(args.instances) if i % n_roll == rank]
        dcfg = DagConfig(instances=args.instances, samples=args.samples, prefix_len=args.prefix, turn_len=args.turn,
                         role_len=args.role, seed=1000 + rank)
        env = MultiAgentDag(cfg.vocab_size, dcfg)
        w = rollout_weights(cfg, dev, n_train, seed=0)
        per_inst = args.prefix + args.samples * (4 * (args.turn + args.role) + 2)
        kv_slots = int(len(inst) * per_inst * 1.15) + 8192
        if args.kv_gb:
            kv_slots = int(args.kv_gb * (1 << 30) / (4 * cfg.layers * cfg.kv_width))
        rows = len(inst) * args.samples * 2
        engine = Engine(cfg, w, kv_slots=kv_slots, max_batch=max(8, 1 << (rows - 1).bit_length()), device=dev,
                        use_graphs=not args.no_graphs)

        class _Env:
            def rollout(self, eng):
                return env.rollout(eng, inst)

        trainer = DisaggRLTrainer("rollout", n_rollout=n_roll, flat=w.flat, push_group=push, engine=engine,
                                  env=_Env(), mb_tokens=args.mb_tokens)
    else:
        engine = None
        if n_train > 1:
            from octopus_b200.parallel.fsdp import FSDPActor

            actor = FSDPActor(cfg, dev, seed=0, group=train_group)
            flat = actor.serve16
        else:
            actor = Actor(cfg, dev, seed=0)
            flat = actor.flat16
        trainer = DisaggRLTrainer("train", n_rollout=n_roll, flat=flat, push_group=push, actor=actor,
                                  mb_tokens=args.mb_tokens)
    for _ in range(args.warmup):
        trainer.step()
    torch.cuda.synchronize()
    ops.check_status(local)
    dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    e0 = dict(engine.stats) if engine is not None else {}
    clocks.start()
    iostats.reset()
    l0 = ops.launches()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    gen, wall, stats = 0, [], []
    start.record()
    for _ in range(args.steps):
        t0 = time.perf_counter()
        st = trainer.step()
        torch.cuda.synchronize()
        wall.append(time.perf_counter() - t0)
        gen += st["generated_tokens"]
        stats.append(st)
    end.record()
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    clk = clocks.stop()
    io = iostats.snapshot()
    launches = ops.launches() - l0
    ms = start.elapsed_time(end)
    ops.check_status(local)
    s0 = stats[-1]
    t = torch.tensor([ms, sum(wall), s0.get("rollout_s", 0.0), s0.get("train_s", 0.0), s0["sync_s"]],
                     dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    sm = torch.tensor([float(gen), float(launches), io["h2d"], io["d2h"], float(s0.get("tree_tokens") or 0),
                       float(s0.get("trained_tokens") or 0)], dtype=torch.float64, device=dev)
    dist.all_reduce(sm, op=dist.ReduceOp.SUM)
    ms, wall_s = float(t[0]), float(t[1])
    gen = float(sm[0])
    value, e2e = gen / (ms / 1000.0), gen / wall_s
    if rank == 0:
        par = (f"disaggregated, one step asynchronous: {n_roll} rollout GPUs (tp1 replicas) + {n_train} trainer GPUs "
               f"(actor {'full-shard fused' if n_train > 1 else 'single GPU'}); rollout k overlaps training on "
               f"rollout k-1")
        out = {
            "metric": METRIC, "value": round(value, 2), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 2), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None if BASELINE_VALUE is None else value / BASELINE_VALUE,
            "dtype": "bf16", "data": "synthetic (uniform random tokens, random-init weights, Bernoulli(0.5) rewards)",
            "config": {"model": args.model + (f"-L{args.layers}" if args.layers else ""),
                       "global_batch": args.instances * args.samples,
                       "seq_len": args.prefix + 4 * (args.turn + args.role), "parallelism": par,
                       "dag": "planner->2 solvers->verifier, prefix mounted zero-copy",
                       "instances": args.instances, "samples": args.samples, "prefix": args.prefix,
                       "turn": args.turn, "staleness": "each rollout trained once, one weight version behind",
                       "tokens_counted": "generated tokens per iteration (each trained once, one iteration later)",
                       "l2": "inputs larger than L2 (7B weights 15 GB, KV > 10 GB per step)"},
            "clocks": clk,
            "e2e": {"value": round(e2e, 2), "unit": "tokens/s", "h2d_bytes_per_step": int(float(sm[2]) / args.steps),
                    "d2h_bytes_per_step": int(float(sm[3]) / args.steps),
                    "api": "octopus_b200.rl.disagg.DisaggRLTrainer.step"},
            "gpu_launches": int(sm[1]),
            "phases_s": {"rollout": round(float(t[2]), 3), "train": round(float(t[3]), 3),
                         "exchange": round(float(t[4]), 4)},
            "engine_per_step": {k: round((engine.stats[k] - e0[k]) / args.steps, 3)
                                for k in ("prefill_s", "decode_s", "decode_steps", "prefill_tokens", "cached_tokens")},
            "trained_tokens_last_step": int(sm[5]), "tree_tokens_last_step": int(sm[4]),
        }
        print(json.dumps(out), flush=True)
    dist.barrier()
    torch.cuda.synchronize()
    if role == "train" and n_train > 1:
        actor.close()
    dist.barrier()
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
