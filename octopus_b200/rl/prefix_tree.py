"""Prefix trees (DAGs once mounts exist) of flat sequences, and their kernel-call plans.

A micro-batch of sequences is trained ONCE over its prefix tree: every shared run of
tokens is stored once (pre-order), the attention of a node sees
``[mounted segments | ancestor path | own rows]`` with bottom-right causality, and the
head scores unique (row, next-token) pairs, so a branch point scores each child's
first token.  Results are exact w.r.t. running every sequence alone.

Mounts: ``mounts[i] = [(at, src, s0, s1), ...]`` means tokens >= ``at`` of sequence i
also attend to tokens ``[s0, s1)`` of sequence ``src`` (keys as src computed them, at
src's positions), plus, transitively, what src itself mounted strictly inside that
range.  A mount point starts a node; sequences share a node only if their tokens and
their mounts so far agree.  Positions follow rule K2: after a mount, the next
position is ``max(own next position, last mounted position + 1)``.

Reference parity (semantics, not code): `octopus/rl/prefix_tree.py:67-166`
(build_tree: nodes, mounted keys, K2 first positions, (pos, label) pairs, flat_pair),
`prefix_tree.py:449-565` (allocate_prefix_groups: prefix-aware first-fit-decreasing
packing with mount units kept whole, cost = tree tokens + KAPPA * query-key pairs).
The construction here is an explicit work-stack over sequence groups with numpy
divergence search; key lists are assembled as tree-row index arrays for the
gathered-key attention kernel.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

Mount = tuple[int, int, int, int]  # (at, src, s0, s1)
KAPPA = 1.0 / 1024.0  # query-key pairs per token of cost (attention vs linear work)


@dataclass
class TreeNode:
    start: int
    end: int
    parent: int
    depth: int
    mounts: tuple  # ((src, s0, s1), ...) mounted at this node's start
    path_segs: list = field(default_factory=list)  # [(start, end)] of ancestors + own, in order


@dataclass
class PrefixTree:
    tokens: np.ndarray          # [T] tree-row tokens
    positions: np.ndarray       # [T] K2 positions
    nodes: list                 # pre-order TreeNode list; node rows tile [0, T)
    mounted: list               # per node: np.ndarray of mounted key rows (incl. inherited)
    pair_row: np.ndarray        # [P] tree row whose hidden state scores pair p
    pair_label: np.ndarray      # [P] next-token label of pair p
    flat_pair: np.ndarray       # [T_flat] pair index of each flat position (-1: not scored / last)
    terminal: np.ndarray        # [n_seq] node where each sequence ends
    seq_len: np.ndarray         # [n_seq]

    @property
    def num_tokens(self) -> int:
        return int(self.tokens.shape[0])

    def path_rows(self, k: int) -> np.ndarray:
        segs = self.nodes[k].path_segs
        if not segs:
            return np.empty(0, dtype=np.int64)
        return np.concatenate([np.arange(a, b, dtype=np.int64) for a, b in segs])

    def flat_to_tree(self) -> np.ndarray:
        return np.concatenate([self.path_rows(int(t)) for t in self.terminal]) if len(self.terminal) else \
            np.empty(0, dtype=np.int64)

    def key_rows(self, k: int, with_mounts: bool = True) -> np.ndarray:
        """Key rows of node k: mounted (optional) + ancestor path + own rows (own last)."""
        path = self.path_rows(k)
        if with_mounts and self.mounted[k].size:
            return np.concatenate([self.mounted[k], path])
        return path

    def attention_pairs(self) -> int:
        tot = 0
        for k, n in enumerate(self.nodes):
            q = n.end - n.start
            keys = len(self.mounted[k]) + sum(b - a for a, b in n.path_segs)
            tot += q * (keys - q) + q * (q + 1) // 2
        return tot


def _first_mismatch(a: np.ndarray, b: np.ndarray) -> int:
    m = min(len(a), len(b))
    d = np.flatnonzero(a[:m] != b[:m])
    return int(d[0]) if d.size else m


def build_tree(flat: np.ndarray, cu, mounts: dict | None = None, scored: np.ndarray | None = None,
               share: bool = True) -> PrefixTree:
    """Prefix tree of sequences flat[cu[i]:cu[i+1]] (see module docstring).  share=False
    gives every sequence its own path (the ordinary packed varlen batch, for checks)."""
    flat = np.asarray(flat)
    cu = [int(x) for x in cu]
    seqs = [flat[a:b] for a, b in zip(cu[:-1], cu[1:])]
    nseq = len(seqs)
    mpts: list[dict] = [dict() for _ in range(nseq)]
    for i, lst in (mounts or {}).items():
        for at, src, s0, s1 in sorted(lst, key=lambda m: m[0]):
            mpts[i][int(at)] = mpts[i].get(int(at), ()) + ((int(src), int(s0), int(s1)),)
    mkeys = [sorted(m) for m in mpts]

    nodes: list[TreeNode] = []
    chunks: list[np.ndarray] = []
    terminal = np.full(nseq, -1, dtype=np.int64)
    total = 0

    def group_children(ids, end):
        groups: dict = {}
        for i in ids:
            if len(seqs[i]) == end:
                continue
            key = (int(seqs[i][end]), mpts[i].get(end, ())) if share else (i,)
            groups.setdefault(key, []).append(i)
        return list(groups.values())

    # work items: (ids, offset, parent); pushed in reverse so pre-order pops first child first
    stack = [(g, 0, -1) for g in reversed(group_children(range(nseq), 0))]
    for i in range(nseq):
        if len(seqs[i]) == 0:
            terminal[i] = -1
    while stack:
        ids, off, parent = stack.pop()
        ref = seqs[ids[0]]
        lim = min(len(seqs[i]) for i in ids) - off
        for i in ids:
            for a in mkeys[i]:
                if a > off:
                    lim = min(lim, a - off)
                    break
        for i in ids[1:]:
            if lim == 0:
                break
            lim = min(lim, _first_mismatch(ref[off:off + lim], seqs[i][off:off + lim]))
        k = len(nodes)
        psegs = list(nodes[parent].path_segs) if parent >= 0 else []
        if lim > 0:
            psegs.append((total, total + lim))
        nodes.append(TreeNode(total, total + lim, parent, nodes[parent].depth + 1 if parent >= 0 else 0,
                              mpts[ids[0]].get(off, ()), psegs))
        chunks.append(ref[off:off + lim])
        total += lim
        end = off + lim
        for i in ids:
            if len(seqs[i]) == end:
                terminal[i] = k
        for g in reversed(group_children(ids, end)):
            stack.append((g, end, k))

    tokens = np.concatenate(chunks) if chunks else np.empty(0, dtype=flat.dtype)
    node_of = np.repeat(np.arange(len(nodes)), [n.end - n.start for n in nodes]) if nodes else \
        np.empty(0, dtype=np.int64)
    tree = PrefixTree(tokens, np.empty(total, dtype=np.int64), nodes, [None] * len(nodes), np.empty(0, np.int64),
                      np.empty(0, np.int64), np.full(len(flat), -1, dtype=np.int64), terminal,
                      np.asarray([len(s) for s in seqs], dtype=np.int64))

    # ---- mounted keys (transitive), memoised per node
    own: dict[int, np.ndarray] = {}
    seq_paths = {}

    def seq_path(src):
        if src not in seq_paths:
            seq_paths[src] = tree.path_rows(int(terminal[src]))
        return seq_paths[src]

    def node_own_keys(k):
        if k not in own:
            parts = [segment(*m) for m in nodes[k].mounts]
            own[k] = np.concatenate(parts) if parts else np.empty(0, dtype=np.int64)
        return own[k]

    def segment(src, s0, s1):
        rows = [seq_path(src)[s0:s1]]
        j = int(terminal[src])
        while j >= 0:
            start_off = sum(b - a for a, b in nodes[j].path_segs) - (nodes[j].end - nodes[j].start)
            if nodes[j].mounts and s0 < start_off < s1:
                rows.append(node_own_keys(j))
            j = nodes[j].parent
        return np.concatenate(rows)

    for k, n in enumerate(nodes):
        inherited = tree.mounted[n.parent] if n.parent >= 0 else np.empty(0, dtype=np.int64)
        ok = node_own_keys(k)
        tree.mounted[k] = np.concatenate([inherited, ok]) if ok.size else inherited

    # ---- K2 positions
    first: dict[int, int] = {}

    def first_pos(k):
        if k in first:
            return first[k]
        n = nodes[k]
        p = first_pos(n.parent) + (nodes[n.parent].end - nodes[n.parent].start) if n.parent >= 0 else 0
        for src, _, s1 in n.mounts:
            last = int(seq_path(src)[s1 - 1])
            j = int(node_of[last])
            p = max(p, first_pos(j) + (last - nodes[j].start) + 1)
        first[k] = p
        return p

    for k, n in enumerate(nodes):
        b = first_pos(k)
        tree.positions[n.start:n.end] = np.arange(b, b + n.end - n.start)

    # ---- (row, label) pairs of scored flat positions
    f2t = tree.flat_to_tree()
    has_next = np.ones(len(flat), dtype=bool) if scored is None else np.asarray(scored, dtype=bool).copy()
    ends = np.asarray(cu[1:], dtype=np.int64) - 1
    has_next[ends[ends >= 0]] = False
    rows = f2t[has_next]
    labels = np.append(flat[1:], 0)[has_next].astype(np.int64)
    if rows.size:
        lo = min(int(labels.min()), 0)  # labels are token ids (>= 0); guard negative ids anyway
        base = int(labels.max()) - lo + 1
        packed = rows.astype(np.int64) * base + (labels - lo)
        uniq, inv = np.unique(packed, return_inverse=True)
        tree.pair_row = uniq // base
        tree.pair_label = uniq % base + lo
        tree.flat_pair[has_next] = inv
    return tree


# ---------------------------------------------------------------------------- plans
@dataclass
class TreePlanHost:
    """Host-side arrays of an attention plan over a (padded) tree."""

    cu_q: np.ndarray
    cu_k: np.ndarray
    key_idx: np.ndarray
    padded_tokens: int


def attention_plan(tree: PrefixTree, with_mounts: bool = True, pad_to: int = 128) -> TreePlanHost:
    """One sequence per node (query rows = node rows, keys = key_rows); padding rows last."""
    cu_q, cu_k, keys = [0], [0], []
    for k, n in enumerate(tree.nodes):
        if n.end == n.start:
            continue
        kr = tree.key_rows(k, with_mounts)
        keys.append(kr)
        cu_q.append(n.end)
        cu_k.append(cu_k[-1] + len(kr))
    T = tree.num_tokens
    Tp = (T + pad_to - 1) // pad_to * pad_to if pad_to else T
    if Tp > T:
        keys.append(np.arange(T, Tp))
        cu_q.append(Tp)
        cu_k.append(cu_k[-1] + Tp - T)
    key_idx = np.concatenate(keys).astype(np.int32) if keys else np.empty(0, np.int32)
    return TreePlanHost(np.asarray(cu_q, np.int32), np.asarray(cu_k, np.int32), key_idx, Tp)


def tree_tokens(seqs: list) -> int:
    """Tokens of the prefix tree of `seqs` (sum of lengths minus shared prefixes)."""
    if not seqs:
        return 0
    order = sorted(range(len(seqs)), key=lambda i: tuple(int(x) for x in seqs[i][:64]))
    srt = [np.asarray(seqs[i]) for i in order]
    srt.sort(key=lambda s: s.tobytes())
    tot = len(srt[0])
    for a, b in zip(srt[:-1], srt[1:]):
        tot += len(b) - _first_mismatch(a, b)
    return int(tot)


def allocate_prefix_groups(seqs: list, cap: int, mounts: dict | None = None, min_groups: int = 1,
                           divisor: int = 1) -> list[list[int]]:
    """Pack sequences into micro-batches of <= cap tree tokens (largest first).

    Sequences linked by mounts stay in one unit (union-find); units are ordered
    lexicographically so shared prefixes land together, then packed first-fit by
    decreasing size.  At least `min_groups` groups are returned and the count is
    rounded up to a multiple of `divisor` (by splitting the largest groups).
    """
    n = len(seqs)
    parent = list(range(n))

    def find(x):
        while parent[x] != x:
            parent[x] = parent[parent[x]]
            x = parent[x]
        return x

    for i, lst in (mounts or {}).items():
        for _, src, _, _ in lst:
            ri, rs = find(i), find(src)
            if ri != rs:
                parent[ri] = rs
    units: dict[int, list[int]] = {}
    for i in range(n):
        units.setdefault(find(i), []).append(i)
    ulist = list(units.values())
    ulist.sort(key=lambda u: np.asarray(seqs[u[0]]).tobytes())
    # merge lexicographic neighbours greedily into prefix groups, then FFD by size
    sized = [(tree_tokens([seqs[i] for i in u]), u) for u in ulist]
    sized.sort(key=lambda x: -x[0])
    bins: list[list[int]] = []
    bin_members: list[list] = []
    for sz, u in sized:
        placed = False
        for b, members in enumerate(bin_members):
            trial = [seqs[i] for i in members + u]
            if tree_tokens(trial) <= cap:
                bin_members[b] = members + u
                placed = True
                break
        if not placed:
            bin_members.append(list(u))
    bins = bin_members
    want = max(min_groups, len(bins))
    if divisor > 1:
        want = (want + divisor - 1) // divisor * divisor
    while len(bins) < want:
        bins.sort(key=lambda b: -tree_tokens([seqs[i] for i in b]))
        big = bins[0]
        if len(big) < 2:
            bins.append([])
            continue
        # split by units: move the second half of the units
        roots = []
        for i in big:
            r = find(i)
            if r not in roots:
                roots.append(r)
        if len(roots) < 2:
            bins.append([])
            continue
        half = set(roots[len(roots) // 2:])
        bins[0] = [i for i in big if find(i) not in half]
        bins.append([i for i in big if find(i) in half])
    bins.sort(key=lambda b: -tree_tokens([seqs[i] for i in b]))
    return bins


def cost(seqs: list) -> float:
    """Micro-batch cost model: tree tokens + KAPPA * causal query-key pairs (flat bound)."""
    pairs = sum(len(s) * (len(s) + 1) // 2 for s in seqs)
    return tree_tokens(seqs) + KAPPA * pairs
