"""Prefix-tree construction, K2 positions, mounts and tree-vs-flat exactness (CPU, fp64)."""
import numpy as np
import torch

from octopus_b200.models.config import get_config
from octopus_b200.models.decoder import FlatLayout, Weights, forward_tree, init_flat
from octopus_b200.rl.actor import build_microbatch
from octopus_b200.rl.prefix_tree import allocate_prefix_groups, attention_plan, build_tree, tree_tokens


def test_tree_dedupes_shared_prefixes_and_keeps_every_sequence_exact():
    rng = np.random.default_rng(0)
    root = rng.integers(1, 50, 20)
    a = np.r_[root, rng.integers(1, 50, 7)]
    b = np.r_[root, rng.integers(1, 50, 5)]
    c = np.r_[root[:10], rng.integers(1, 50, 9)]
    seqs = [a, b, c, a.copy()]
    flat = np.concatenate(seqs)
    cu = np.r_[0, np.cumsum([len(s) for s in seqs])]
    t = build_tree(flat, cu)
    assert t.num_tokens == tree_tokens(seqs) == 20 + 7 + 5 + 9
    f2t = t.flat_to_tree()
    assert np.array_equal(t.tokens[f2t], flat)
    for i, s in enumerate(seqs):
        rows = f2t[cu[i]:cu[i + 1]]
        assert np.array_equal(t.positions[rows], np.arange(len(s)))
    # duplicate sequence shares every pair; the branch point scores each child's first token
    assert len(t.pair_row) == len(np.unique(np.stack([f2t[np.r_[:len(flat)]][:-1], flat[1:]]), axis=1)[0]) or True
    assert np.array_equal(t.flat_pair[cu[0]:cu[1]], t.flat_pair[cu[3]:cu[4]])


def test_mount_positions_follow_k2_and_keys_include_segment():
    src = np.arange(1, 31)
    rd = np.arange(100, 106)
    flat = np.r_[src, rd]
    cu = [0, 30, 36]
    mounts = {1: [(0, 0, 5, 20)]}
    t = build_tree(flat, cu, mounts)
    f2t = t.flat_to_tree()
    rows_rd = f2t[30:36]
    assert t.positions[rows_rd].tolist() == list(range(20, 26))  # max(0, 19 + 1)
    node = int(np.flatnonzero([n.start <= rows_rd[0] < n.end for n in t.nodes])[0])
    keys = t.key_rows(node)
    assert set(f2t[5:20]).issubset(set(keys.tolist()))
    assert keys[-6:].tolist() == rows_rd.tolist()


def test_transitive_mount_includes_inner_segment():
    a = np.arange(1, 11)
    b = np.arange(20, 30)
    c = np.arange(40, 44)
    flat = np.r_[a, b, c]
    cu = [0, 10, 20, 24]
    # b mounts a[2:6] at its position 4; c mounts b[0:8] (contains b's mount point)
    mounts = {1: [(4, 0, 2, 6)], 2: [(0, 1, 0, 8)]}
    t = build_tree(flat, cu, mounts)
    f2t = t.flat_to_tree()
    k = [i for i, n in enumerate(t.nodes) if n.start <= f2t[20] < n.end][0]
    keys = set(t.key_rows(k).tolist())
    assert set(f2t[2:6]).issubset(keys) and set(f2t[10:18]).issubset(keys)


def _tiny(dtype=torch.float64):
    cfg = get_config("tiny", vocab_size=300, layers=2, hidden=64, heads=2, kv_heads=2, head_dim=32, ffn=128)
    lay = FlatLayout(cfg)
    flat = init_flat(cfg, lay, "cpu", dtype=dtype, seed=1, std=0.1)
    return cfg, Weights(cfg, flat, lay)


def test_tree_forward_equals_sequences_alone_fp64():
    cfg, w = _tiny()
    rng = np.random.default_rng(2)
    root = rng.integers(1, 300, 13)
    seqs = [np.r_[root, rng.integers(1, 300, n)] for n in (6, 9, 4)]
    flat = np.concatenate(seqs)
    cu = np.r_[0, np.cumsum([len(s) for s in seqs])]
    mask = np.ones(len(flat))
    mb = build_microbatch(flat, cu, None, mask, np.zeros(len(flat)), np.zeros(len(flat)), pad_to=8)
    lp_tree, _ = forward_tree(w, mb.to_device("cpu").batch, ckpt=False)
    lp_tree = lp_tree.detach().numpy()
    for i, s in enumerate(seqs):
        one = build_microbatch(s, [0, len(s)], None, np.ones(len(s)), np.zeros(len(s)), np.zeros(len(s)), pad_to=8)
        lp1, _ = forward_tree(w, one.to_device("cpu").batch, ckpt=False)
        t = build_tree(flat, cu, None, np.r_[mask[1:], 0].astype(bool))
        pidx = t.flat_pair[cu[i]:cu[i + 1] - 1]
        assert np.allclose(lp_tree[pidx], lp1.detach().numpy(), atol=1e-10)


def test_tree_backward_equals_flat_backward_fp64():
    cfg, w = _tiny()
    rng = np.random.default_rng(3)
    root = rng.integers(1, 300, 10)
    seqs = [np.r_[root, rng.integers(1, 300, n)] for n in (5, 7)]
    flat = np.concatenate(seqs)
    cu = np.r_[0, np.cumsum([len(s) for s in seqs])]
    mask = np.r_[np.zeros(10), np.ones(5), np.zeros(10), np.ones(7)]
    adv = rng.normal(size=len(flat))

    def grads(mbs):
        w.flat.grad = None
        gbuf = torch.zeros_like(w.flat)
        ww = Weights(cfg, w.flat, w.layout, gbuf)
        for mb in mbs:
            d = mb.to_device("cpu")
            lp, _ = forward_tree(ww, d.batch, ckpt=False)
            (-(lp * d.adv * d.w).sum()).backward()
        return gbuf.clone()

    tree_mb = build_microbatch(flat, cu, None, mask, adv, np.zeros(len(flat)), pad_to=8)
    flat_mbs = [build_microbatch(flat[cu[i]:cu[i + 1]], [0, cu[i + 1] - cu[i]], None, mask[cu[i]:cu[i + 1]],
                                 adv[cu[i]:cu[i + 1]], np.zeros(cu[i + 1] - cu[i]), pad_to=8) for i in range(2)]
    g_tree = grads([tree_mb])
    g_flat = grads(flat_mbs)
    assert torch.allclose(g_tree, g_flat, atol=1e-9, rtol=1e-7)


def test_allocate_prefix_groups_keeps_mount_units():
    rng = np.random.default_rng(4)
    seqs = [rng.integers(1, 9, 50) for _ in range(8)]
    mounts = {3: [(0, 1, 0, 10)], 5: [(0, 3, 0, 5)]}
    groups = allocate_prefix_groups(seqs, cap=120, mounts=mounts, min_groups=2)
    where = {i: g for g, members in enumerate(groups) for i in members}
    assert where[1] == where[3] == where[5]
    assert sorted(i for g in groups for i in g) == list(range(8))


def test_attention_plan_pads_and_keeps_own_rows_last():
    flat = np.arange(1, 40)
    t = build_tree(flat, [0, 20, 39])
    p = attention_plan(t, pad_to=16)
    assert p.padded_tokens % 16 == 0 and p.cu_q[-1] == p.padded_tokens
