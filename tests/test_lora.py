"""LoRA on CPU: the adapter op's gradients equal autograd of the dense formula, the base
gets none; a LoRA actor step moves only the adapters and the merged serving weights are
W + s B A; PEFT export round trip; the zero adapter is the base model; targets map."""
import numpy as np
import pytest
import torch

from octopus_b200 import ops
from octopus_b200.models.config import get_config
from octopus_b200.models.lora import LoRA, LoRAConfig, lora_targets, merge, zero_adapter
from octopus_b200.rl.actor import LoRAActor, OptimConfig, build_microbatch


def test_lora_linear_grads():
    torch.manual_seed(0)
    x = torch.randn(10, 16, dtype=torch.float64, requires_grad=True)
    W = torch.randn(12, 16, dtype=torch.float64)
    A = torch.randn(4, 16, dtype=torch.float64)
    B = torch.randn(12, 4, dtype=torch.float64)
    A.main_grad = torch.zeros_like(A)
    B.main_grad = torch.zeros_like(B)
    r = torch.randn(10, 12, dtype=torch.float64, requires_grad=True)
    y = ops.linear(x, W, None, residual=r, lora=(A, B, 0.5))
    g = torch.randn_like(y)
    y.backward(g)
    xr = x.detach().clone().requires_grad_(True)
    Ar, Br = A.clone().requires_grad_(True), B.clone().requires_grad_(True)
    rr = r.detach().clone().requires_grad_(True)
    yr = xr @ W.t() + 0.5 * (xr @ Ar.t()) @ Br.t() + rr
    yr.backward(g)
    assert torch.allclose(y, yr)
    assert torch.allclose(x.grad, xr.grad) and torch.allclose(r.grad, rr.grad)
    assert torch.allclose(A.main_grad, Ar.grad) and torch.allclose(B.main_grad, Br.grad)


def test_lora_actor_step_and_merge(tmp_path):
    cfg = get_config("tiny", layers=2)
    act = LoRAActor(cfg, "cpu", lora=LoRAConfig(r=8, alpha=16), dtype=torch.float32, ckpt=True,
                    optim=OptimConfig(lr=1e-2))
    base0 = act.base16.clone()
    assert torch.allclose(act.serving.flat, base0)  # B = 0: the serving weights are the base
    rng = np.random.default_rng(0)
    toks = rng.integers(1, cfg.vocab_size, 48)
    mb = build_microbatch(toks, [0, 48], None, np.ones(48, np.float32), rng.normal(size=48).astype(np.float32),
                          np.zeros(48, np.float32), pad_to=8)
    act.train_step([mb])
    assert torch.equal(act.base16, base0)              # the base is frozen
    assert float(act.lora.grad.abs().sum()) > 0
    # serving = base + s B A
    t = "layers.1.gu_w"
    A, B = act.lora.t[f"{t}.A"], act.lora.t[f"{t}.B"]
    want = act.base[t] + act.lora.lcfg.scale * (B @ A)
    assert torch.allclose(act.serving[t], want, atol=1e-5)
    assert float(B.abs().sum()) > 0
    # PEFT round trip
    act.lora.save_peft(str(tmp_path / "ad"))
    other = LoRA(cfg, LoRAConfig(r=8, alpha=16), "cpu", torch.float32, seed=9)
    other.load_peft(str(tmp_path / "ad"))
    assert torch.allclose(other.flat16, act.lora.flat16)


def test_zero_adapter_and_targets(tmp_path):
    cfg = get_config("tiny", layers=1)
    zero_adapter(cfg, str(tmp_path / "z"), LoRAConfig(r=4, alpha=4))
    lo = LoRA(cfg, LoRAConfig(r=4, alpha=4), "cpu", torch.float32)
    lo.load_peft(str(tmp_path / "z"))
    assert float(sum(lo.t[f"layers.0.{t}.B"].abs().sum() for t in ("qkv_w", "o_w", "gu_w", "down_w"))) == 0.0
    assert lora_targets("all-linear") == ("qkv_w", "o_w", "gu_w", "down_w")
    assert lora_targets(["q_proj", "down_proj"]) == ("qkv_w", "down_w")
    with pytest.raises(ValueError):
        lora_targets(["lm_head"])
