"""Hybrid-model serving on CPU (fp64): the engine's logprobs of sampled tokens equal a whole-
sequence hybrid forward; a continuation from a cursor equals one pass over the whole history
(the recurrent and conv states are kept per cursor), also for rows cut early by a stop token
or a smaller max_new_tokens in a mixed batch; mounts reach attention layers only and run;
released cursors answer 404."""
import numpy as np
import pytest
import torch

from octopus_b200.models.config import get_config
from octopus_b200.models.hybrid import HybridConfig, HybridWeights, hybrid_forward
from octopus_b200.rl.actor import build_microbatch
from octopus_b200.serving.engine import CursorNotFound, GenInput
from octopus_b200.serving.hybrid_engine import HybridEngine


def _setup(kind="gdn"):
    base = get_config("tiny", layers=4, vocab_size=512)
    hw = HybridWeights(HybridConfig(base, kind=kind, pattern="LLAL", lin_heads=2, lin_dim=32), "cpu",
                       dtype=torch.float64, seed=3, std=0.05)
    return hw, HybridEngine(hw, kv_slots=8000, max_batch=8, device="cpu")


def _full_logprobs(hw, seq):
    n = len(seq)
    mb = build_microbatch(np.asarray(seq), [0, n], None, np.ones(n, np.float32), np.zeros(n, np.float32),
                          np.zeros(n, np.float32), pad_to=8)
    d = mb.to_device("cpu")
    with torch.no_grad():
        lp, _ = hybrid_forward(hw, d.batch)
    out = np.full(n, np.nan)
    # pair p scores flat position row+1 (tree rows = flat rows for one sequence)
    out[np.asarray(mb.pair_row) + 1] = lp.numpy()
    return out


def _check(hw, history, new_tokens, lps):
    full = _full_logprobs(hw, list(history) + list(new_tokens))
    want = full[len(history):]
    assert np.allclose(np.asarray(lps), want, atol=1e-8), (np.asarray(lps), want)


@pytest.mark.parametrize("kind", ["gdn", "gla"])
def test_generate_matches_whole_sequence(kind):
    hw, eng = _setup(kind)
    rng = np.random.default_rng(0)
    p = rng.integers(1, 512, 23).tolist()
    o = eng.generate([GenInput(p, max_new_tokens=6, cursor_id="a")])[0]
    _check(hw, p, o.output_ids, o.output_logprobs)
    # continue from the cursor: the history is prompt + reply (the last token has no KV yet)
    q = rng.integers(1, 512, 5).tolist()
    o2 = eng.generate([GenInput(q, cursor="a", max_new_tokens=4, cursor_id="b")])[0]
    _check(hw, p + o.output_ids + q, o2.output_ids, o2.output_logprobs)


def test_mixed_batch_and_stop_tokens_keep_exact_states():
    hw, eng = _setup()
    rng = np.random.default_rng(1)
    p1, p2 = rng.integers(1, 512, 17).tolist(), rng.integers(1, 512, 29).tolist()
    probe = eng.generate([GenInput(p1, max_new_tokens=8, rid=11, keep_cursor=False)])[0]
    stop = probe.output_ids[2]
    outs = eng.generate([GenInput(p1, max_new_tokens=8, rid=11, cursor_id="s", stop_ids=(stop,)),
                         GenInput(p2, max_new_tokens=3, rid=12, cursor_id="m")])
    assert outs[0].output_ids == probe.output_ids[:outs[0].output_ids.index(stop) + 1]
    assert len(outs[1].output_ids) == 3
    for o, p, cid in ((outs[0], p1, "s"), (outs[1], p2, "m")):
        q = rng.integers(1, 512, 4).tolist()
        c = eng.generate([GenInput(q, cursor=cid, max_new_tokens=3, keep_cursor=False)])[0]
        _check(hw, p + o.output_ids + q, c.output_ids, c.output_logprobs)


def test_mount_runs_and_cursor_release():
    hw, eng = _setup()
    rng = np.random.default_rng(2)
    a = eng.generate([GenInput(rng.integers(1, 512, 20).tolist(), max_new_tokens=2, cursor_id="src")])[0]
    b = eng.generate([GenInput(rng.integers(1, 512, 9).tolist(), max_new_tokens=2, cursor_id="rd")])[0]
    o = eng.generate([GenInput(rng.integers(1, 512, 3).tolist(), cursor="rd", mount=[("src", 2, 12)],
                               max_new_tokens=3, keep_cursor=False)])[0]
    assert len(o.output_ids) == 3 and np.isfinite(o.output_logprobs).all()
    eng.release_cursor("rd")
    with pytest.raises(CursorNotFound):
        eng.generate([GenInput([5, 6], cursor="rd", max_new_tokens=1)])
    assert a.cursor == "src" and b.cursor == "rd"


@pytest.mark.gpu
def test_hybrid_engine_gpu_close_to_forward():
    """bf16 on the sm_100a kernels (7B attention shapes, GDN layers 2 x 128): the engine's
    logprobs of its sampled tokens, and of a cursor continuation, are close to the
    whole-sequence hybrid forward."""
    dev = torch.device("cuda", 0)
    hw = HybridWeights(HybridConfig(get_config("qwen2.5-7b", layers=4), kind="gdn", pattern="LLAL", lin_heads=2,
                                    lin_dim=128), dev, dtype=torch.bfloat16, seed=3)
    eng = HybridEngine(hw, kv_slots=1 << 14, max_batch=8, device=dev)
    rng = np.random.default_rng(0)
    p = rng.integers(1, 50000, 40).tolist()
    o = eng.generate([GenInput(p, max_new_tokens=6, cursor_id="a")])[0]
    q = rng.integers(1, 50000, 7).tolist()
    o2 = eng.generate([GenInput(q, cursor="a", max_new_tokens=4, keep_cursor=False)])[0]
    for hist, new, lps in ((p, o.output_ids, o.output_logprobs), (p + o.output_ids + q, o2.output_ids,
                                                                  o2.output_logprobs)):
        seq = list(hist) + list(new)
        n = len(seq)
        mb = build_microbatch(np.asarray(seq), [0, n], None, np.ones(n, np.float32), np.zeros(n, np.float32),
                              np.zeros(n, np.float32), pad_to=8)
        with torch.no_grad():
            lp, _ = hybrid_forward(hw, mb.to_device(dev).batch)
        full = np.full(n, np.nan)
        full[np.asarray(mb.pair_row) + 1] = lp.float().cpu().numpy()
        assert np.abs(np.asarray(lps) - full[len(hist):]).max() < 0.1
    torch.cuda.synchronize()
