"""Workflow glue: episodes of the agent runtime -> per-token training rows.

An episode is the runtime's record (`CursorRuntime.run`): its request rows (reply id,
thread, prompt and completion tokens, in order), the outcome `y`, and optionally the
graded branches.  The engine's interaction records (`Engine.records`, reply id ->
tokens, completion length, behaviour logprobs, parent cursor, mounts) give the token
sequences.  Per group of episodes of one task:

1. R = 2y - 1 and leave-one-out advantages (`group.group_step`), branch credit;
2. the exported leaves: the last reply of every thread that no child thread continues;
3. single ownership (`group.assign_threads`): every completion is trained by exactly
   one leaf, adopted requests carry their own thread's advantage as a span;
4. one training row per leaf: the leaf's full token sequence, loss mask on the
   completions it owns (the inherited prefix is masked out), per-token advantage
   (row advantage + span deltas), behaviour logprobs, and its read mounts (the leaf's
   reply chain's mounts, with the mounted source mapped to the row holding those rows,
   or to an extra unscored row for a source that is no leaf's ancestor);
5. a group whose rewards are all equal carries no advantage and is dropped
   (`has_variance`, the dynamic filter).

Rows of a group form one mount unit; `rows_to_microbatches` packs units into
prefix-tree micro-batches under a token cap.

Reference parity (behaviour): `octopus/rl/workflow.py:38-448` (EpisodeAgent.run,
plan_group_rewards, _apply_plan, spool integration, has_variance filter),
`octopus/rl/prefix_tree.py:568-622` (read export: record_reads / seq_mounts).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from ..runtime.core import branch_key
from ..serving.cursor_store import PLACEHOLDER
from .group import _is_child_thread, assign_threads, group_step, has_variance


@dataclass
class TrainRow:
    rid: str
    tokens: np.ndarray
    loss_mask: np.ndarray
    adv: np.ndarray
    behav: np.ndarray
    mounts: list = field(default_factory=list)   # [(at, source rid, s0, s1)]
    version: int = 0
    reward: float = 0.0


def leaves_of(requests: list[dict]) -> list[str]:
    """Reply ids of the exported leaves: each thread's last reply, unless a child thread
    starts after it (that reply forked; its branches continue it)."""
    last: dict[str, int] = {}
    first: dict[str, int] = {}
    for i, r in enumerate(requests):
        th = r.get("thread") or "main"
        last[th] = i
        first.setdefault(th, i)
    out = []
    for th, i in last.items():
        forked = any(_is_child_thread(th, c) and first[c] > i for c in first)
        if not forked:
            out.append(requests[i]["id"])
    order = {r["id"]: k for k, r in enumerate(requests)}
    return sorted(out, key=order.get)


def _chain(rid: str, records: dict) -> list[str]:
    out = []
    while rid is not None and rid in records:
        out.append(rid)
        rid = records[rid].get("parent")
    return out[::-1]


def episode_rows(episode: dict, records: dict) -> list[TrainRow]:
    """Training rows of one episode whose R / A_main / A_branch are already set."""
    reqs = [(r["id"], r.get("thread") or "main", int(r["prompt_tokens"]), int(r["completion_tokens"]))
            for r in episode["requests"]]
    leaves = leaves_of(episode["requests"])
    owners = assign_threads(leaves, {**episode, "requests": reqs})
    rows = []
    for lid in leaves:
        rec = records[lid]
        own = owners[lid]
        n = len(rec["tokens"])
        mask = np.zeros(n, np.float32)
        adv = np.full(n, own["adv"], np.float32)
        beh = np.zeros(n, np.float32)
        chain = _chain(lid, records)
        if own["own_start"] is not None:
            # completions of this leaf's reply chain from its first owned request on
            for rid in chain:
                rr = records[rid]
                a, b = rr["prompt_len"], rr["prompt_len"] + rr["completion"]
                if a >= own["own_start"]:
                    mask[a:b] = 1.0
                    beh[a:b] = rr["logprobs"][: b - a]
        for a, b, d in own["spans"]:
            adv[a:b] += d
        read_adv = episode.get("read_adv") or {}
        for rid in chain:  # a read reply with a read control: its completion gets r_reader - r_control more
            if rid in read_adv:
                rr = records[rid]
                adv[rr["prompt_len"]: rr["prompt_len"] + rr["completion"]] += read_adv[rid]["v"]
        # mounted rows are placeholders in the engine's sequence; the prefix tree takes the
        # sequence without them plus (at, source, s0, s1) mounts in that coordinate system
        toks = rec["tokens"]
        keep = toks != PLACEHOLDER
        before = np.cumsum(~keep)  # placeholders up to and including each index
        mounts = []
        for rid in chain:
            for at, src, s0, s1 in records[rid]["mounts"]:
                at_s = at - (int(before[at - 1]) if at > 0 else 0)
                mounts.append((at_s, src, s0, s1))
        rows.append(TrainRow(lid, toks[keep].astype(np.int64), mask[keep], adv[keep], beh[keep], mounts,
                             rec.get("version", 0), own["reward"]))
    return rows


def _source_range(src: str, s0: int, s1: int, records: dict) -> tuple[int, int]:
    """[s0, s1) of a source cursor's rows in its placeholder-free coordinates."""
    toks = records[src]["tokens"]
    ph = toks[:s1] == PLACEHOLDER
    if ph[s0:s1].any():
        raise NotImplementedError("mounting rows that are themselves mounted (transitive mount) from a training row")
    k = int(ph[:s0].sum())
    return s0 - k, s1 - k


def plan_group_rewards(episodes: list[dict], records: dict, branch_credit: str = "outcome", gate=None,
                       filter_zero_variance: bool = True, read_rewards=None) -> list[TrainRow]:
    """Rows of one group (episodes of the same task); [] when the group is filtered."""
    if filter_zero_variance and not has_variance([float(e["y"]) for e in episodes]):
        return []
    for e in episodes:  # every branch thread gets a branch record (ungraded ones: outcome / gate defaults)
        have = {b["key"] for b in e.get("branches") or []}
        for r in e["requests"]:
            th = r.get("thread") or "main"
            if th != "main" and not th.startswith("readctl/") and th != "control" and branch_key(th) not in have:
                e.setdefault("branches", []).append({"key": branch_key(th)})
                have.add(branch_key(th))
    group_step(episodes, branch_credit=branch_credit, gate=gate, read_rewards=read_rewards)
    return [row for e in episodes for row in episode_rows(e, records)]


def _source_row(src: str, rows: list[TrainRow], records: dict) -> int | None:
    for k, r in enumerate(rows):
        if src == r.rid or src in _chain(r.rid, records):
            return k
    return None


def unit_sequences(rows: list[TrainRow], records: dict):
    """(seqs, mounts {seq: [(at, src seq, s0, s1)]}, masks, behs, advs) of one mount unit;
    mounted sources that are no row's ancestor become extra unscored sequences."""
    seqs = [r.tokens for r in rows]
    masks = [r.loss_mask for r in rows]
    behs = [r.behav for r in rows]
    advs = [r.adv for r in rows]
    extra: dict[str, int] = {}
    mounts: dict[int, list] = {}
    for j, r in enumerate(rows):
        for at, src, s0, s1 in r.mounts:
            k = _source_row(src, rows, records)
            if k is None:
                if src not in extra:
                    toks = records[src]["tokens"]
                    toks = toks[toks != PLACEHOLDER].astype(np.int64)
                    extra[src] = len(seqs)
                    seqs.append(toks)
                    masks.append(np.zeros(len(toks), np.float32))
                    behs.append(np.zeros(len(toks), np.float32))
                    advs.append(np.zeros(len(toks), np.float32))
                k = extra[src]
            a, b = _source_range(src, s0, s1, records)
            mounts.setdefault(j, []).append((at, k, a, b))
    return seqs, mounts, masks, behs, advs


def rows_to_microbatches(units: list[list[TrainRow]], records: dict, token_cap: int, build):
    """Pack mount units (groups) into prefix-tree micro-batches of <= token_cap flat tokens."""
    packed, cur, cur_n = [], [], 0
    for u in units:
        seqs, mounts, masks, behs, advs = unit_sequences(u, records)
        n = sum(len(s) for s in seqs)
        if cur and cur_n + n > token_cap:
            packed.append(cur)
            cur, cur_n = [], 0
        cur.append((seqs, mounts, masks, behs, advs))
        cur_n += n
    if cur:
        packed.append(cur)
    mbs = []
    for g in packed:
        flat, cu, mounts, mask, beh, adv = [], [0], {}, [], [], []
        for seqs, m, masks, behs, advs in g:
            base = len(cu) - 1
            for s in seqs:
                flat.append(s)
                cu.append(cu[-1] + len(s))
            for j, lst in m.items():
                mounts[base + j] = [(at, base + src, s0, s1) for at, src, s0, s1 in lst]
            mask += list(masks)
            beh += list(behs)
            adv += list(advs)
        mbs.append(build(np.concatenate(flat), cu, mounts, np.concatenate(mask), np.concatenate(adv),
                         np.concatenate(beh)))
    return mbs
