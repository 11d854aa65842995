"""Shard layout of the tensor-parallel engine on CPU: one layer computed from the TP
shards of `tp` virtual ranks (rank-order reduction of the row-parallel partials) equals
the full layer; the reshard copies reproduce the slices; row sizes of the fused kernels."""
import torch

from octopus_b200.models.config import get_config
from octopus_b200.models.decoder import FlatLayout, Weights, init_flat
from octopus_b200.ops import reference as ref
from octopus_b200.parallel.tp import TPWeights, reference_layer, shard_dims, tp_rows


def _weights(cfg):
    lay = FlatLayout(cfg)
    flat = init_flat(cfg, lay, "cpu", dtype=torch.float32, seed=0)
    return Weights(cfg, flat, lay)


def _attn(q, k, v, hq, hkv, pos):
    T, D = q.shape[0], 128
    qh, kh, vh = q.view(T, hq, D), k.view(T, hkv, D), v.view(T, hkv, D)
    cu = torch.tensor([0, T])
    o, _ = ref.gather_attention(qh, kh, vh, cu, cu, torch.arange(T), D ** -0.5)
    return o.reshape(T, hq * D).float()


def test_tp_layer_matches_full_layer():
    cfg = get_config("tiny-tp")
    w = _weights(cfg)
    torch.manual_seed(0)
    x = torch.randn(24, cfg.hidden)
    pos = torch.arange(24)
    full = reference_layer(cfg, w, 1, x, pos, _attn)
    for tp in (2, 4):
        got = reference_layer(cfg, w, tp, x, pos, _attn)
        assert torch.allclose(got, full, rtol=1e-4, atol=1e-4), tp


def test_tp_weights_slices():
    cfg = get_config("tiny-tp")
    w = _weights(cfg)
    for r in range(2):
        sd = shard_dims(cfg, 2, r)
        tw = TPWeights(cfg, w, sd, "cpu")
        qkv = tw.t["layers.1.qkv_w"]
        assert torch.equal(qkv[:sd.q_loc], w["layers.1.qkv_w"][r * sd.q_loc:(r + 1) * sd.q_loc])
        k0 = cfg.q_width + r * sd.kv_loc
        assert torch.equal(qkv[sd.q_loc:sd.q_loc + sd.kv_loc], w["layers.1.qkv_w"][k0:k0 + sd.kv_loc])
        assert torch.equal(tw.t["layers.0.down_w"], w["layers.0.down_w"][:, r * sd.f:(r + 1) * sd.f])
        gu = tw.t["layers.0.gu_w"]
        assert torch.equal(gu[sd.f:], w["layers.0.gu_w"][cfg.ffn + r * sd.f:cfg.ffn + (r + 1) * sd.f])
        assert torch.equal(tw.head, w.head[sd.col_base:sd.col_base + sd.vocab_limit])
        b = tw.t["layers.0.qkv_b"]
        assert torch.equal(b[sd.q_loc + sd.kv_loc:], w["layers.0.qkv_b"][cfg.q_width + cfg.kv_width + r * sd.kv_loc:
                                                                       cfg.q_width + cfg.kv_width + (r + 1) * sd.kv_loc])


def test_tp_rows():
    assert [tp_rows(n) for n in (1, 8, 9, 33, 100, 128, 129, 1000)] == [8, 8, 16, 64, 128, 128, 256, 1024]
