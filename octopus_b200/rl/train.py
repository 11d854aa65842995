"""RL trainer entry point.

    python -m octopus_b200.rl.train [--config grpo.yaml] [key=value ...]
    torchrun --nproc-per-node 8 -m octopus_b200.rl.train --config grpo.yaml rollout.tp=2

One process per GPU.  Per step: rollout (colocated engine, or a tensor-parallel group of
`rollout.tp` GPUs), group credit + prefix-tree micro-batches, the actor update (ZeRO-
sharded over all ranks with fused peer-memory collectives), weight sync; then a JSON
step line (`<run>/steps.jsonl` and stdout), a recover checkpoint every
`checkpoint.recover_every` steps (followed by the rollout spool commit) and HF
safetensors every `checkpoint.save_every` steps.  A run resumes from its recover
checkpoint.  `OCTOPUS_LIVE_ENV` (MB_TOKENS, ...) is re-read every step.

Reference parity (behaviour): `octopus/rl/train.py:55-137` (derived settings, episode
settings snapshot, dataset, trainer with spool commit after the recover checkpoint,
dynamic filter).
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

DEFAULT_CONFIG = os.path.join(os.path.dirname(os.path.abspath(__file__)), "grpo.yaml")


def _dist_init(device):
    import torch.distributed as dist
    from datetime import timedelta

    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1 and not dist.is_initialized():
        backend = "nccl" if device.type == "cuda" else "gloo"
        kw = {"device_id": device} if device.type == "cuda" else {}
        dist.init_process_group(backend, timeout=timedelta(seconds=900), **kw)
    return world


def build_disagg(cfg, device, world: int, rank: int):
    """(trainer, actor or None, engine or None, spool, trainer group) of a disaggregated run (dense model,
    rollout TP 1, no LoRA): rollout ranks get an engine over their own weight copy and their
    share of the environment, trainer ranks the actor (full-shard over the trainer ranks)."""
    import torch

    from ..models.config import get_config
    from ..serving.engine import Engine
    from .actor import Actor, OptimConfig
    from .disagg import DisaggRLTrainer, make_groups, rollout_weights, split_roles
    from .loss import PPOConfig
    from .spool import Spool

    a = cfg.actor
    if cfg.rollout.tp > 1 or a.lora_rank > 0 or cfg.model.path:
        raise SystemExit("rl.disaggregate: dense random-init models, rollout.tp 1, no LoRA")
    mcfg = get_config(cfg.model.preset, **({"layers": cfg.model.layers} if cfg.model.layers else {}))
    dtype = torch.bfloat16 if device.type == "cuda" else torch.float32
    n_roll = split_roles(world, cfg.rl.rollout_gpus)
    n_train = world - n_roll
    train_group, push = make_groups(world, n_roll)
    spool = Spool(cfg.rl.spool) if cfg.rl.spool else None
    if rank < n_roll:
        w = rollout_weights(mcfg, device, n_train, dtype=dtype, seed=cfg.seed)
        kv_slots = int(cfg.rollout.kv_gb * (1 << 30) / (4 * mcfg.layers * mcfg.kv_width))
        engine = Engine(mcfg, w, kv_slots=kv_slots, max_batch=cfg.rollout.max_batch, device=device)
        env = _make_env(cfg, mcfg, engine, rank, n_roll)
        tr = DisaggRLTrainer("rollout", n_rollout=n_roll, flat=w.flat, push_group=push, engine=engine, env=env,
                             mb_tokens=a.mb_tokens, report=True)
        return tr, None, engine, spool, train_group
    optim = OptimConfig(lr=a.lr, betas=(a.beta1, a.beta2), eps=a.eps, weight_decay=a.weight_decay,
                        max_grad_norm=a.gradient_clipping)
    ppo = PPOConfig(eps_clip=a.eps_clip, eps_clip_higher=a.eps_clip_higher, behav_imp_weight_cap=a.behav_imp_weight_cap,
                    reuse_train_logp=a.reuse_train_logp)
    if n_train > 1:
        from ..parallel.fsdp import FSDPActor

        actor = FSDPActor(mcfg, device, optim=optim, ppo=ppo, seed=cfg.seed, dtype=dtype, group=train_group,
                          fused=a.fused_collectives and device.type == "cuda")
        flat = actor.serve16
    else:
        actor = Actor(mcfg, device, optim=optim, ppo=ppo, seed=cfg.seed, dtype=dtype, ckpt=a.gradient_checkpointing)
        flat = actor.flat16
    tr = DisaggRLTrainer("train", n_rollout=n_roll, flat=flat, push_group=push, actor=actor, mb_tokens=a.mb_tokens,
                         report=True)
    return tr, actor, None, spool, train_group


def _make_env(cfg, mcfg, engine, rep: int, replicas: int):
    """The environment of rollout replica `rep` of `replicas` (its share of the tasks)."""
    from ..envs.dag import DagConfig, MultiAgentDag

    if cfg.rl.kind == "dag":
        inst = [i for i in range(cfg.rl.batch_size) if i % replicas == rep]
        dag = MultiAgentDag(mcfg.vocab_size, DagConfig(instances=cfg.rl.batch_size, samples=cfg.rl.n_samples,
                                                       prefix_len=cfg.rl.dag_prefix, turn_len=cfg.rl.dag_turn,
                                                       temperature=cfg.rollout.temperature,
                                                       seed=cfg.seed * 1000 + rep))

        class _Env:
            def rollout(self, eng):
                return dag.rollout(eng, inst)

        return _Env()
    if cfg.rl.kind == "search":
        return _search_env(cfg, engine, rep, replicas)
    if cfg.rl.kind == "swe":
        return _swe_env(cfg, engine, rep, replicas)
    raise SystemExit(f"rl.kind {cfg.rl.kind!r}: dag, search or swe")


def build(cfg, device):
    """(trainer, actor, engine, env, spool, tp_rank) for a run config."""
    import torch
    import torch.distributed as dist

    from ..models.config import get_config
    from ..models.decoder import load_hf
    from ..parallel.fsdp import ShardedActor
    from ..serving.engine import Engine
    from .actor import Actor, OptimConfig
    from .loss import PPOConfig
    from .spool import Spool
    from .trainer import RLTrainer, TrainerConfig

    world = dist.get_world_size() if dist.is_initialized() else 1
    rank = dist.get_rank() if dist.is_initialized() else 0
    from ..models.hybrid import hybrid_config

    hc = hybrid_config(cfg.model.preset, cfg.model.layers)
    mcfg = hc.base if hc is not None else get_config(cfg.model.preset,
                                                     **({"layers": cfg.model.layers} if cfg.model.layers else {}))
    a = cfg.actor
    optim = OptimConfig(lr=a.lr, betas=(a.beta1, a.beta2), eps=a.eps, weight_decay=a.weight_decay,
                        max_grad_norm=a.gradient_clipping)
    ppo = PPOConfig(eps_clip=a.eps_clip, eps_clip_higher=a.eps_clip_higher, behav_imp_weight_cap=a.behav_imp_weight_cap,
                    reuse_train_logp=a.reuse_train_logp)
    dtype = torch.bfloat16 if device.type == "cuda" else torch.float32
    if hc is not None:
        if cfg.rollout.tp > 1:
            raise SystemExit("hybrid presets: no rollout TP")
        from .hybrid_actor import HybridActor, HybridLoRAActor

        if a.lora_rank > 0:
            actor = HybridLoRAActor(hc, device, r=a.lora_rank, alpha=a.lora_alpha, optim=optim, ppo=ppo, seed=cfg.seed,
                                    dtype=dtype, ckpt=a.gradient_checkpointing)
        else:
            actor = HybridActor(hc, device, optim=optim, ppo=ppo, seed=cfg.seed, dtype=dtype,
                                ckpt=a.gradient_checkpointing)
        if world > 1:  # replicated data parallelism: one all-reduce of every gradient per step
            from ..parallel.dp import DataParallel

            DataParallel(actor).attach_actor()
    elif a.lora_rank > 0:
        from ..models.lora import LoRAConfig, lora_targets
        from .actor import LoRAActor

        targets = lora_targets(a.lora_targets if "," not in a.lora_targets else a.lora_targets.split(","))
        actor = LoRAActor(mcfg, device, lora=LoRAConfig(a.lora_rank, a.lora_alpha, targets), optim=optim, ppo=ppo,
                          seed=cfg.seed, dtype=dtype, ckpt=a.gradient_checkpointing)
        if world > 1:
            from ..parallel.dp import DataParallel

            DataParallel(actor).attach_actor()
    elif world > 1 and a.full_shard:
        from ..parallel.fsdp import FSDPActor

        actor = FSDPActor(mcfg, device, optim=optim, ppo=ppo, seed=cfg.seed, dtype=dtype,
                          fused=a.fused_collectives and device.type == "cuda", gather_weights=a.gather_weights)
    elif world > 1 and a.sharded:
        actor = ShardedActor(mcfg, device, optim=optim, ppo=ppo, seed=cfg.seed, dtype=dtype,
                             ckpt=a.gradient_checkpointing, fused=a.fused_collectives and device.type == "cuda")
    else:
        actor = Actor(mcfg, device, optim=optim, ppo=ppo, seed=cfg.seed, dtype=dtype, ckpt=a.gradient_checkpointing)
    chunk_tokens = a.chunk_tokens
    if not chunk_tokens and os.environ.get("OCTOPUS_CHUNK_MAJOR", "0") == "1":  # the reference's host switch
        chunk_tokens = int(os.environ.get("OCTOPUS_CHUNK_TOKENS", "32768"))
    actor.set_memory(a.ckpt_block, int(a.act_gpu_gb * (1 << 30)) if a.act_gpu_gb >= 0 else None,
                     chunk_tokens=chunk_tokens, seq_tile=a.seq_tile)
    if cfg.model.path:
        base = getattr(actor, "base", actor.weights)
        load_hf(base.dense if hc is not None and hasattr(base, "dense") else base, cfg.model.path)
        if hc is not None:
            _load_hybrid_linear(actor, cfg.model.path)
        actor.reload_master()
        if a.lora_rank > 0:
            actor.optimizer_merge()
    tp = max(1, cfg.rollout.tp)
    rep, tp_rank = rank // tp, rank % tp
    group = None
    if tp > 1:
        for r in range(world // tp):
            g = dist.new_group(list(range(r * tp, (r + 1) * tp)))
            if r == rep:
                group = g
    kv_slots = int(cfg.rollout.kv_gb * (1 << 30) / (4 * mcfg.layers * mcfg.kv_width // tp))
    if hc is not None:
        from ..serving.hybrid_engine import HybridEngine

        engine = HybridEngine(actor.hw, kv_slots=kv_slots, max_batch=cfg.rollout.max_batch, device=device)
    elif tp > 1:
        from ..serving.tp_engine import TPEngine

        engine = TPEngine(mcfg, actor.weights, group=group, kv_slots=kv_slots, max_batch=cfg.rollout.max_batch,
                          device=device)
    else:
        engine = Engine(mcfg, actor.weights, kv_slots=kv_slots, max_batch=cfg.rollout.max_batch, device=device)
    replicas = world // tp
    spool = Spool(cfg.rl.spool) if cfg.rl.spool else None
    env = _make_env(cfg, mcfg, engine, rep, replicas)
    trainer = RLTrainer(actor, engine, env, TrainerConfig(mb_tokens=a.mb_tokens, mb_shard=(tp_rank, tp)),
                        sync_fn=engine.sync_weights if tp > 1 else None)
    return trainer, actor, engine, env, spool, tp_rank


def _search_env(cfg, engine, rep, replicas):
    from ..envs.search.agent import SearchWorkspace, search_defaults
    from ..envs.search.reward import search_outcome
    from ..envs.search.service import make_retrieval
    from ..rl.group import search_gate
    from ..serving.chat import ChatTokenizer
    from ..serving.local import ChatService
    from .agent_env import AgentEnv

    if not cfg.rl.search_questions:
        raise SystemExit("rl.kind=search needs rl.search_questions (JSONL of {qid, question, answer[, corpus]})")
    rows = [json.loads(x) for x in open(cfg.rl.search_questions) if x.strip()]
    rows = [r for i, r in enumerate(rows) if i % replicas == rep]
    corpus_path = os.environ.get("OCTOPUS_SEARCH_CORPUS", "")
    corpus = [json.loads(x) for x in open(corpus_path)] if corpus_path else [
        {"docid": r["qid"], "title": r["question"], "text": str(r.get("context", ""))} for r in rows]
    # OCTOPUS_SEARCH_BACKEND=dense: document embeddings OCTOPUS_SEARCH_EMBEDDINGS (glob of pickles), query
    # encoder OCTOPUS_SEARCH_ENCODER (local checkpoint path)
    retrieval = make_retrieval(corpus, os.environ.get("OCTOPUS_SEARCH_BACKEND", "bm25"),
                               os.environ.get("OCTOPUS_SEARCH_EMBEDDINGS", ""),
                               os.environ.get("OCTOPUS_SEARCH_ENCODER", ""),
                               os.environ.get("OCTOPUS_SEARCH_DEVICE", "cpu"))
    search_defaults()
    tok = ChatTokenizer.from_dir(cfg.model.path) if cfg.model.path else ChatTokenizer.tiny()
    svc = ChatService(engine, tok)
    return AgentEnv(svc, rows, lambda t: SearchWorkspace(retrieval, t["question"]),
                    lambda t, ans: search_outcome(ans, t["answer"], t["question"]), n_samples=cfg.rl.n_samples,
                    batch_size=max(1, cfg.rl.batch_size // replicas), branch_credit=cfg.rl.branch_credit,
                    gate=search_gate if cfg.rl.branch_credit == "gate" else None,
                    filter_zero_variance=cfg.rl.filter_zero_variance)


def _observability(engine, before: dict, device) -> dict:
    """Per-step serving and memory figures for the step log: prefix-cache hit rate (rows
    reused from the radix cache or cursors / rows prefilled or reused), requests, KV pool
    usage, peak device memory and host RSS."""
    import torch

    d = {k: engine.stats.get(k, 0) - before.get(k, 0) for k in ("cached_tokens", "prefill_tokens", "requests")}
    tot = d["cached_tokens"] + d["prefill_tokens"]
    out = {"cache_hit_rate": round(d["cached_tokens"] / tot, 4) if tot else None, "requests": d["requests"]}
    try:
        ls = engine.load_stats()
        out["kv_usage"] = round(float(ls.get("token_usage", 0.0)), 4)
    except Exception:  # noqa: BLE001  (engines without a pool report)
        pass
    if device.type == "cuda":
        out["peak_gpu_gb"] = round(torch.cuda.max_memory_allocated(device) / 2**30, 3)
    try:
        import psutil

        out["host_rss_gb"] = round(psutil.Process().memory_info().rss / 2**30, 3)
    except ImportError:
        pass
    return out


def _load_hybrid_linear(actor, path):
    """Linear-layer tensors of a hybrid checkpoint written by HybridActor.save_hf."""
    f = os.path.join(path, "hybrid_linear.safetensors")
    if not os.path.exists(f):
        raise SystemExit(f"{path}: no hybrid_linear.safetensors for the hybrid preset's linear layers")
    from safetensors.torch import load_file

    st = load_file(f)
    import torch

    hw = actor.base if hasattr(actor, "lora") else actor.hw  # LoRA: the frozen base
    with torch.no_grad():
        for k, t in list(hw.t.items()) + list(hw.fp32.items()):
            t.copy_(st[k].to(t.dtype))


def _swe_env(cfg, engine, rep, replicas):
    """SWE plan episodes (envs.swe.rl): the task rows of this replica, bundled when asked,
    graded by their hidden tests in local sandboxed copies."""
    from ..envs.swe.containers import LocalExec
    from ..envs.swe.rl import swe_agent_env
    from ..envs.swe.taskset import build_bundles, load_rows, select_task_specs
    from ..serving.chat import ChatTokenizer
    from ..serving.local import ChatService

    if not cfg.rl.swe_tasks:
        raise SystemExit("rl.kind=swe needs rl.swe_tasks (JSONL task rows or a directory of them)")
    specs = select_task_specs(load_rows(cfg.rl.swe_tasks))
    if cfg.rl.swe_bundle > 1:
        specs = build_bundles(specs, cfg.rl.swe_bundle, seed=cfg.seed)
    specs = [s for i, s in enumerate(specs) if i % replicas == rep]
    if not specs:
        raise SystemExit(f"rl.swe_tasks {cfg.rl.swe_tasks}: no task with a local repository for this replica")
    tok = ChatTokenizer.from_dir(cfg.model.path) if cfg.model.path else ChatTokenizer.tiny()
    return swe_agent_env(ChatService(engine, tok), specs, LocalExec(sandbox=True), n_samples=cfg.rl.n_samples,
                         batch_size=max(1, cfg.rl.batch_size // replicas), branch_credit=cfg.rl.branch_credit,
                         timeout=cfg.rl.swe_timeout, filter_zero_variance=cfg.rl.filter_zero_variance)


def _push_weights(actor, cfg, run_dir: str) -> dict:
    """Weight sync to remote rollout hosts (rollout.push_hosts): the adapter (LoRA actors)
    or the HF weights of this version, written under run_dir/push/v<version> and copied
    to <push_dir>/v<version> on every host (rl.adapter_push: tar over ssh with retries)."""
    from ..models.decoder import save_hf
    from .adapter_push import push_adapter

    src = os.path.join(run_dir, "push", f"v{actor.version}")
    if hasattr(actor, "lora"):
        actor.lora.save_peft(src, base_model=cfg.model.path)
    else:
        save_hf(actor.weights, src)
    hosts = [h.strip() for h in cfg.rollout.push_hosts.split(",") if h.strip()]
    dest = os.path.join(cfg.rollout.push_dir or "octopus_weights", f"v{actor.version}")
    return push_adapter(src, hosts, dest)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m octopus_b200.rl.train")
    ap.add_argument("--config", default=DEFAULT_CONFIG)
    ap.add_argument("--cpu", action="store_true", help="run on CPU (tiny models, tests)")
    ap.add_argument("overrides", nargs="*", help="dotted key=value overrides")
    args = ap.parse_args(argv)

    import torch
    import torch.distributed as dist

    from . import checkpoint
    from . import config as C
    from ..models.decoder import save_hf

    cfg = C.load(args.config, args.overrides)
    C.set_derived_settings(cfg)
    local = int(os.environ.get("LOCAL_RANK", "0"))
    device = torch.device("cpu") if args.cpu or not torch.cuda.is_available() else torch.device("cuda", local)
    if device.type == "cuda":
        torch.cuda.set_device(device)
    world = _dist_init(device)
    rank = dist.get_rank() if world > 1 else 0
    run_dir = os.path.join(cfg.checkpoint.dir or "runs", cfg.experiment_name, cfg.trial_name)
    if rank == 0:
        os.makedirs(run_dir, exist_ok=True)
        C.save_settings(os.path.join(run_dir, "episode_settings.json"))
        with open(os.path.join(run_dir, "config.json"), "w") as f:
            json.dump(cfg.to_dict(), f, indent=1)
    if world > 1 and cfg.rl.disaggregate:
        return _main_disagg(cfg, device, world, rank, run_dir)
    trainer, actor, engine, env, spool, tp_rank = build(cfg, device)
    step0 = 0
    if checkpoint.exists(run_dir):
        state = checkpoint.load(actor, run_dir)
        step0 = int(state["step"])
        engine.bump_version()
        if hasattr(engine, "sync_weights"):
            engine.sync_weights()
    log = open(os.path.join(run_dir, "steps.jsonl"), "a") if rank == 0 else None
    for step in range(step0, cfg.total_steps):
        live = C.live_env()
        if "MB_TOKENS" in live:
            trainer.cfg.mb_tokens = live["MB_TOKENS"]
        t0 = time.time()
        seen = dict(engine.stats)
        if device.type == "cuda":
            torch.cuda.reset_peak_memory_stats(device)
        st = trainer.step()
        row = {"step": step + 1, "time": round(time.time() - t0, 3), "version": actor.version,
               **{k: (round(v, 6) if isinstance(v, float) else v) for k, v in st.items()
                  if isinstance(v, (int, float))}, **_observability(engine, seen, device)}
        if rank == 0:
            line = json.dumps(row)
            print(line, flush=True)
            log.write(line + "\n")
            log.flush()
        if cfg.rollout.push_hosts and rank == 0:
            _push_weights(actor, cfg, run_dir)
        if cfg.checkpoint.recover_every and (step + 1) % cfg.checkpoint.recover_every == 0:
            checkpoint.save(actor, run_dir, step + 1, {"step": step + 1}, spool=spool)
        if cfg.checkpoint.save_every and (step + 1) % cfg.checkpoint.save_every == 0 and rank == 0:
            out_dir = os.path.join(run_dir, f"hf-step{step + 1}")
            actor.save_hf(out_dir) if hasattr(actor, "save_hf") else save_hf(actor.weights, out_dir)
    if world > 1:
        dist.barrier()
        if hasattr(engine, "close"):
            engine._graphs.clear()
            engine.close()
        if hasattr(actor, "close"):
            actor.close()
        dist.destroy_process_group()
    return 0


def _main_disagg(cfg, device, world: int, rank: int, run_dir: str) -> int:
    """Training loop of a disaggregated run: every rank steps the loop; trainer ranks keep the
    recover checkpoints, the first trainer rank writes HF weights, rank 0 the step log (its
    rollout numbers plus the first trainer rank's, prefixed train_ where both have a key)."""
    import torch
    import torch.distributed as dist

    from . import checkpoint
    from ..models.decoder import save_hf

    trainer, actor, engine, spool, group = build_disagg(cfg, device, world, rank)
    n_roll = trainer.n_rollout
    step0 = 0
    if actor is not None and checkpoint.exists(run_dir):
        step0 = int(checkpoint.load(actor, run_dir, group=group)["step"])
    s = torch.tensor([step0], dtype=torch.int64, device=device)
    dist.broadcast(s, src=n_roll)  # every rank resumes at the trainer's step
    step0 = int(s.item())
    if step0:
        trainer.push_weights()  # the rollout ranks start from the restored weights
    log = open(os.path.join(run_dir, "steps.jsonl"), "a") if rank == 0 else None
    for step in range(step0, cfg.total_steps):
        t0 = time.time()
        st = trainer.step()
        if rank == 0:
            row = {"step": step + 1, "time": round(time.time() - t0, 3),
                   **{k: (round(v, 6) if isinstance(v, float) else v) for k, v in st.items()
                      if isinstance(v, (int, float))}}
            line = json.dumps(row)
            print(line, flush=True)
            log.write(line + "\n")
            log.flush()
        if actor is not None:
            if cfg.checkpoint.recover_every and (step + 1) % cfg.checkpoint.recover_every == 0:
                checkpoint.save(actor, run_dir, step + 1, {"step": step + 1}, spool=spool, group=group)
            if cfg.checkpoint.save_every and (step + 1) % cfg.checkpoint.save_every == 0 and rank == n_roll:
                save_hf(actor.weights, os.path.join(run_dir, f"hf-step{step + 1}"))
    dist.barrier()
    if engine is not None and hasattr(engine, "close"):
        engine._graphs.clear()
    if hasattr(actor, "close"):
        actor.close()
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
