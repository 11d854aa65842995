"""Hybrid-model training on CPU: the hybrid actor's step moves the dense, linear-layer and
fp32 gate / conv parameters under one global clip; the colocated hybrid engine serves the
updated weights (its logprobs equal a fresh whole-sequence forward); chunk-major training
gives the whole-tree gradients; extra state round-trips; the trainer CLI runs a hybrid
preset for a step, saves hybrid_linear.safetensors and resumes."""
import json

import numpy as np
import torch

from octopus_b200.models.hybrid import HybridConfig, hybrid_config, hybrid_forward
from octopus_b200.models.config import get_config
from octopus_b200.rl.actor import OptimConfig, build_microbatch
from octopus_b200.rl.hybrid_actor import HybridActor
from octopus_b200.serving.engine import GenInput
from octopus_b200.serving.hybrid_engine import HybridEngine


def _mb(seed=0, V=512):
    rng = np.random.default_rng(seed)
    root = rng.integers(1, V, 14)
    seqs = [np.r_[root, rng.integers(1, V, 9)], np.r_[root, rng.integers(1, V, 6)]]
    flat = np.concatenate(seqs)
    n = len(flat)
    return build_microbatch(flat, np.r_[0, np.cumsum([len(s) for s in seqs])], None, np.ones(n, np.float32),
                            rng.normal(size=n).astype(np.float32), np.zeros(n, np.float32), pad_to=8)


def _actor(dtype=torch.float64):
    hc = HybridConfig(get_config("tiny", layers=4, vocab_size=512), kind="gdn", pattern="LLAL", lin_heads=2,
                      lin_dim=32)
    return HybridActor(hc, "cpu", optim=OptimConfig(lr=1e-3, max_grad_norm=0.5), dtype=dtype, seed=1)


def test_step_moves_every_group_and_engine_serves_it():
    act = _actor()
    eng = HybridEngine(act.hw, kv_slots=4000, max_batch=8, device="cpu")
    dense0 = act.flat16.clone()
    lin0 = {k: t.clone() for k, t in act.hw.t.items()}
    p0 = {k: p.detach().clone() for k, p in act.hw.fp32.items()}
    st = act.train_step([_mb()])
    assert torch.isfinite(st["loss"]) and float(st["grad_norm"]) > 0
    assert not torch.equal(act.flat16, dense0)
    assert all(not torch.equal(act.hw.t[k], lin0[k]) for k in lin0 if k.endswith(("lin_qkv", "lin_out")))
    assert all(not torch.equal(act.hw.fp32[k].detach(), p0[k]) for k in p0)
    # the engine reads the updated tensors in place
    rng = np.random.default_rng(3)
    p = rng.integers(1, 512, 12).tolist()
    o = eng.generate([GenInput(p, max_new_tokens=4, keep_cursor=False)])[0]
    seq = p + o.output_ids
    n = len(seq)
    mb = build_microbatch(np.asarray(seq), [0, n], None, np.ones(n, np.float32), np.zeros(n, np.float32),
                          np.zeros(n, np.float32), pad_to=8)
    with torch.no_grad():
        lp, _ = hybrid_forward(act.hw, mb.to_device("cpu").batch)
    full = np.full(n, np.nan)
    full[np.asarray(mb.pair_row) + 1] = lp.numpy()
    assert np.allclose(o.output_logprobs, full[len(p):], atol=1e-8)


def test_chunk_major_step_equals_whole_tree():
    a, b = _actor(), _actor()
    b.set_memory(chunk_tokens=8)
    mb = _mb(2)
    a.zero_grad()
    b.zero_grad()
    a.forward_backward([mb])
    b.forward_backward([mb])
    assert torch.allclose(a.grad, b.grad, rtol=1e-7, atol=1e-10)
    for k, t in a.hw.t.items():
        assert torch.allclose(t.main_grad, b.hw.t[k].main_grad, rtol=1e-7, atol=1e-10)


def test_extra_state_round_trip():
    a, b = _actor(), _actor()
    a.train_step([_mb()])
    b.load_extra_state(a.extra_state())
    for k in a.hw.t:
        assert torch.equal(a.hw.t[k], b.hw.t[k]) and torch.equal(a.lin_m[k], b.lin_m[k])
    for k in a.hw.fp32:
        assert torch.equal(a.hw.fp32[k].detach(), b.hw.fp32[k].detach())


def test_presets():
    assert hybrid_config("qwen2.5-7b") is None
    hc = hybrid_config("hybrid-7b", layers=8)
    assert hc.base.layers == 8 and hc.pattern == "LLLA" and hc.ba_rows % 8 == 0


def test_train_cli_hybrid(tmp_path, monkeypatch):
    from octopus_b200.envs import dag
    from octopus_b200.rl import train

    orig = dag.DagConfig.__init__

    def small(self, *a, **kw):
        orig(self, *a, **kw)
        self.prefix_len, self.turn_len, self.role_len = 32, 8, 4

    monkeypatch.setattr(dag.DagConfig, "__init__", small)
    args = ["--cpu", "model.preset=tiny-hybrid", "rl.kind=dag", "rl.batch_size=2", "rl.n_samples=2",
            "rollout.kv_gb=0.05", "rollout.max_batch=16", "actor.mb_tokens=65536", f"checkpoint.dir={tmp_path}",
            "checkpoint.save_every=1", "total_steps=1"]
    assert train.main(args) == 0
    run = tmp_path / "octopus-b200" / "run0"
    assert (run / "hf-step1" / "hybrid_linear.safetensors").exists()
    assert train.main(args[:-1] + ["total_steps=2"]) == 0
    rows = [json.loads(x) for x in open(run / "steps.jsonl")]
    assert [r["step"] for r in rows] == [1, 2]


def test_hybrid_actor_gpu_step():
    """One hybrid training step on the sm_100a kernels (7B attention shapes, 4 layers): finite
    loss, every parameter group moves, the engine generates from the updated weights."""
    import pytest

    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    dev = torch.device("cuda", 0)
    act = HybridActor(hybrid_config("hybrid-7b", layers=4), dev, optim=OptimConfig(lr=1e-4), seed=2)
    eng = HybridEngine(act.hw, kv_slots=1 << 14, max_batch=8, device=dev)
    p0 = {k: p.detach().clone() for k, p in act.hw.fp32.items()}
    q0 = act.hw.t["layers.0.lin_qkv"].clone()
    st = act.train_step([_mb(4, V=50000)])
    torch.cuda.synchronize()
    assert torch.isfinite(st["loss"]) and float(st["grad_norm"]) > 0
    assert not torch.equal(act.hw.t["layers.0.lin_qkv"], q0)
    assert all(not torch.equal(act.hw.fp32[k].detach(), p0[k]) for k in p0)
    o = eng.generate([GenInput(list(range(100, 140)), max_new_tokens=4, keep_cursor=False)])[0]
    assert len(o.output_ids) == 4 and np.isfinite(o.output_logprobs).all()


test_hybrid_actor_gpu_step = __import__("pytest").mark.gpu(test_hybrid_actor_gpu_step)


def test_server_cli_builds_from_hybrid_checkpoint(tmp_path):
    """A hybrid checkpoint written by the actor loads into the server's hybrid engine; the
    server CLI builds a dense engine and its app."""
    from octopus_b200.serving.server import build_engine, main

    act = HybridActor(hybrid_config("tiny-hybrid"), "cpu", dtype=torch.float32, seed=4)
    act.train_step([_mb(5, V=4096)])
    act.save_hf(str(tmp_path / "ck"))
    eng, _ = build_engine("tiny-hybrid", str(tmp_path / "ck"), kv_gb=0.01, max_batch=8, device="cpu")
    assert type(eng).__name__ == "HybridEngine"
    for k in ("layers.0.lin_qkv", "layers.1.lin_ba"):
        assert torch.equal(eng.hw.t[k], act.hw.t[k])
    assert torch.equal(eng.hw.fp32["layers.0.A_log"].detach(), act.hw.fp32["layers.0.A_log"].detach())
    assert torch.equal(eng.w.flat, act.flat16)
    assert main(["--preset", "tiny", "--kv-gb", "0.01", "--max-batch", "8", "--device", "cpu", "--check"]) == 0


def _dp_rank(rank, world, port, q):
    import os
    from datetime import timedelta

    import torch.distributed as dist

    from octopus_b200.parallel.dp import DataParallel

    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        act = _actor()
        DataParallel(act).attach_actor()
        act.zero_grad()
        act.forward_backward([_mb(10 + rank)])
        act.optimizer_step()
        q.put((rank, act.flat16.clone().numpy(), {k: t.clone().numpy() for k, t in act.hw.t.items()},
               {k: p.detach().clone().numpy() for k, p in act.hw.fp32.items()}))
    finally:
        dist.destroy_process_group()


def test_hybrid_data_parallel_matches_one_process():
    """Two gloo ranks, one micro-batch each, equal the one-process step over both."""
    import socket

    import torch.multiprocessing as mp

    ref = _actor()
    ref.zero_grad()
    ref.forward_backward([_mb(10), _mb(11)])
    ref.optimizer_step()
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_dp_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict((r, rest) for r, *rest in (q.get(timeout=300) for _ in procs))
    for p in procs:
        p.join(timeout=60)
    for r in (0, 1):
        flat, lin, fp = got[r]
        assert np.allclose(flat, ref.flat16.numpy(), rtol=1e-9, atol=1e-12)
        for k, t in ref.hw.t.items():
            assert np.allclose(lin[k], t.numpy(), rtol=1e-9, atol=1e-12), k
        for k, p in ref.hw.fp32.items():
            assert np.allclose(fp[k], p.detach().numpy(), rtol=1e-9, atol=1e-12), k


def test_hybrid_lora_actor():
    """Hybrid LoRA: only the adapters train (the frozen base has no gradient buffers), the
    serving copy equals base + s B A, and the hybrid forward on the serving copy equals the
    base forward with the adapters; the trainer CLI runs a LoRA step on the hybrid preset."""
    from octopus_b200.rl.hybrid_actor import HybridLoRAActor

    hc = HybridConfig(get_config("tiny", layers=4, vocab_size=512), kind="gdn", pattern="LLAL", lin_heads=2,
                      lin_dim=32)
    act = HybridLoRAActor(hc, "cpu", r=4, alpha=8.0, optim=OptimConfig(lr=1e-2), dtype=torch.float64, seed=1)
    assert act.base.grad is None and not any(hasattr(t, "main_grad") for t in act.base.t.values())
    base0 = act.base.dense.flat.clone()
    assert torch.equal(act.hw.dense.flat, base0)  # B = 0: serving = base
    act.train_step([_mb()])
    assert torch.equal(act.base.dense.flat, base0) and float(act.lora.grad.abs().sum()) > 0
    name = "layers.0.lin_qkv"
    A, B = act.lora.t[f"{name}.A"], act.lora.t[f"{name}.B"]
    assert float(B.abs().sum()) > 0
    assert torch.allclose(act.hw.t[name], act.base.t[name] + act.lora.scale * (B @ A), atol=1e-12)
    mb = _mb(7).to_device("cpu")
    with torch.no_grad():
        lp_serve, _ = hybrid_forward(act.hw, mb.batch)
        lp_lora, _ = hybrid_forward(act.base, mb.batch, lora=act.lora)
    assert torch.allclose(lp_serve, lp_lora, atol=1e-9)


def test_train_cli_hybrid_lora(tmp_path, monkeypatch):
    from octopus_b200.envs import dag
    from octopus_b200.rl import train

    orig = dag.DagConfig.__init__

    def small(self, *a, **kw):
        orig(self, *a, **kw)
        self.prefix_len, self.turn_len, self.role_len = 32, 8, 4

    monkeypatch.setattr(dag.DagConfig, "__init__", small)
    args = ["--cpu", "model.preset=tiny-hybrid", "rl.kind=dag", "rl.batch_size=2", "rl.n_samples=2",
            "rollout.kv_gb=0.05", "rollout.max_batch=16", "actor.mb_tokens=65536", "actor.lora_rank=8",
            f"checkpoint.dir={tmp_path}", "checkpoint.save_every=1", "total_steps=1"]
    assert train.main(args) == 0
    assert train.main(args[:-1] + ["total_steps=2"]) == 0
    rows = [json.loads(x) for x in open(tmp_path / "octopus-b200" / "run0" / "steps.jsonl")]
    assert [r["step"] for r in rows] == [1, 2]


@__import__("pytest").mark.gpu
def test_hybrid_lora_actor_gpu_step():
    """One hybrid LoRA step on the sm_100a kernels (r = 8): the adapters move, the serving copy
    changes, the engine generates from it."""
    from octopus_b200.rl.hybrid_actor import HybridLoRAActor

    dev = torch.device("cuda", 0)
    act = HybridLoRAActor(hybrid_config("hybrid-7b", layers=4), dev, r=8, alpha=16.0, optim=OptimConfig(lr=1e-3),
                          seed=2)
    eng = HybridEngine(act.hw, kv_slots=1 << 14, max_batch=8, device=dev)
    s0 = act.hw.t["layers.0.lin_qkv"].clone()
    st = act.train_step([_mb(4, V=50000)])
    torch.cuda.synchronize()
    assert torch.isfinite(st["loss"]) and float(st["grad_norm"]) > 0
    assert not torch.equal(act.hw.t["layers.0.lin_qkv"], s0)
    o = eng.generate([GenInput(list(range(100, 140)), max_new_tokens=4, keep_cursor=False)])[0]
    assert len(o.output_ids) == 4 and np.isfinite(o.output_logprobs).all()
