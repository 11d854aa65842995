"""Data-parallel balance: split a step's groups into per-episode items weighted by their
prefix-tree tokens and partition them over ranks longest-first.

An all-plan group is split into per-episode dispatch items (an episode's sequences
stay together: they share a tree); each item's weight is its prefix-tree size (the
work it costs), and items are assigned largest first to the rank with the least work
so far (LPT).  This replaces an equal-count partition, which loads ranks unevenly
when trees differ in size.

Reference parity (behaviour): `octopus/rl/dp_balance.py:47-131`.
"""
from __future__ import annotations

import heapq

from .prefix_tree import tree_tokens


def item_weights(items: list[list]) -> list[int]:
    """items: per episode, its token sequences -> prefix-tree tokens of each."""
    return [tree_tokens(seqs) for seqs in items]


def longest_first(weights: list[int], world: int) -> list[list[int]]:
    """Assign item indices to `world` ranks, largest first to the least-loaded rank."""
    heap = [(0, r) for r in range(world)]
    out: list[list[int]] = [[] for _ in range(world)]
    for i in sorted(range(len(weights)), key=lambda i: -weights[i]):
        load, r = heapq.heappop(heap)
        out[r].append(i)
        heapq.heappush(heap, (load + weights[i], r))
    return out


def partition(items: list[list], world: int) -> tuple[list[list[int]], list[int]]:
    w = item_weights(items)
    parts = longest_first(w, world)
    return parts, [sum(w[i] for i in p) for p in parts]


def take_rows(parts: list[list[int]], rank: int) -> list[int]:
    return parts[rank]
