"""Top-p / top-k sampling on CPU: the filter keeps the top-k set and the smallest nucleus,
top_k >= vocab (or 0) means no top-k, sampled tokens stay inside the kept set and follow the
renormalised distribution, logprobs are under the full tempered distribution, draws are
per-row deterministic; the engine and chat service pass the fields through."""
import numpy as np
import pytest
import torch

from octopus_b200 import ops
from octopus_b200.ops.core import _uniform, filter_logits


def test_filter_logits_sets():
    z = torch.log(torch.tensor([[0.5, 0.2, 0.15, 0.1, 0.05]], dtype=torch.float64))
    assert filter_logits(z, 1.0, 2).tolist() == [[True, True, False, False, False]]
    assert filter_logits(z, 0.6, 0).tolist() == [[True, True, False, False, False]]  # 0.5 < 0.6 <= 0.7
    assert filter_logits(z, 0.45, 0).tolist() == [[True, False, False, False, False]]
    assert filter_logits(z, 0.01, 0).tolist() == [[True, False, False, False, False]]  # top token always kept
    # top-p on the top-k renormalised mass: 0.588, 0.235, 0.176
    assert filter_logits(z, 0.85, 3).tolist() == [[True, True, True, False, False]]
    assert filter_logits(z, 0.8, 3).tolist() == [[True, True, False, False, False]]
    assert filter_logits(z, 1.0, 5).all() and filter_logits(z, 1.0, 99).all()


def test_uniform_is_per_row_deterministic():
    a = _uniform(7, torch.tensor([3, 4, 5]), 100)
    b = _uniform(7, torch.tensor([5]), 100)
    assert torch.equal(a[2], b[0]) and (a > 0).all() and (a < 1).all()
    assert not torch.equal(a[0], a[1]) and not torch.equal(_uniform(8, torch.tensor([3]), 100)[0], a[0])
    u = _uniform(1, torch.arange(64), 4096).flatten()
    assert abs(float(u.mean()) - 0.5) < 0.01 and abs(float((u < 0.1).double().mean()) - 0.1) < 0.01


def test_sample_respects_filters_and_distribution():
    torch.manual_seed(0)
    H, V = 16, 40
    W = torch.randn(V, H, dtype=torch.float64)
    h = torch.randn(1, H, dtype=torch.float64).repeat(4000, 1)
    z = (h[:1] @ W.t())[0]
    streams = torch.arange(4000)
    tok, lp = ops.sample(h, W, 1.0, 3, streams, V, top_p=1.0, top_k=3)
    top3 = set(z.topk(3).indices.tolist())
    assert set(tok.tolist()) <= top3
    p3 = torch.softmax(z[list(sorted(top3))], 0)
    freq = torch.tensor([(tok == t).double().mean().item() for t in sorted(top3)])
    assert float((freq - p3).abs().max()) < 0.03
    full = torch.log_softmax(z, 0)
    assert torch.allclose(lp.double(), full[tok], atol=1e-6)
    tok1, _ = ops.sample(h[:8], W, 1.0, 3, None, V, top_k=1)
    assert (tok1 == z.argmax()).all()
    tokp, _ = ops.sample(h[:200], W, 0.7, 5, streams[:200], V, top_p=0.5)
    keep = filter_logits((z / 0.7)[None], 0.5, 0)[0]
    assert keep[tokp].all()
    a, _ = ops.sample(h[:5], W, 1.0, 9, streams[:5], V, top_p=0.9)
    b, _ = ops.sample(h[2:5], W, 1.0, 9, streams[2:5], V, top_p=0.9)
    assert torch.equal(a[2:], b)  # a row's draw does not depend on the batch


def test_engine_top_k_one_is_greedy():
    from octopus_b200.serving.engine import GenInput
    from test_engine_cpu import tiny_engine

    _, _, eng = tiny_engine()
    rng = np.random.default_rng(0)
    prompt = rng.integers(1, 500, 30).tolist()
    g = eng.generate([GenInput(prompt, max_new_tokens=6, temperature=1.0, top_k=1, keep_cursor=False)])[0]
    cold = eng.generate([GenInput(prompt, max_new_tokens=6, temperature=1e-4, keep_cursor=False)])[0]
    assert g.output_ids == cold.output_ids
    n = eng.generate([GenInput(prompt, max_new_tokens=6, temperature=1.0, top_p=0.3, keep_cursor=False)])[0]
    assert len(n.output_ids) == 6 and all(np.isfinite(n.output_logprobs))


def test_service_fields():
    from octopus_b200.serving.local import _top_k
    from octopus_b200.serving.server import generate_input

    assert _top_k(None) == 0 and _top_k(-1) == 0 and _top_k(20) == 20
    g = generate_input({"input_ids": [1, 2], "sampling_params": {"max_new_tokens": 4, "top_p": 0.95, "top_k": 20}})
    assert g.top_p == pytest.approx(0.95) and g.top_k == 20


def test_noise_depends_on_the_whole_row_stream():
    """Row streams are (request id << 32 | position): two requests at the same position must
    draw different noise (the high 32 bits enter the row key)."""
    import torch

    from octopus_b200.ops.core import _uniform

    s = torch.tensor([(7 << 32) | 100, (8 << 32) | 100, (7 << 32) | 101], dtype=torch.int64)
    u = _uniform(3, s, 64)
    assert not torch.equal(u[0], u[1]) and not torch.equal(u[0], u[2])
    assert float(u.min()) > 0.0 and float(u.max()) < 1.0
