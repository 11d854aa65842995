"""Synthetic multi-agent DAG environment: planner -> 2 parallel solvers -> verifier.

Each DAG instance has a shared random prefix (the task) that every agent mounts
zero-copy.  Per sample of an instance:

  planner   mounts the prefix, reads a role prompt, writes ``turn`` tokens
  solver k  forks the planner (continues its cursor: shares the planner's KV as a
            prefix), reads its role prompt, writes ``turn`` tokens   (k = 1, 2)
  verifier  mounts the prefix and both solvers' outputs (K2 positions), reads its
            role prompt, writes ``turn`` tokens

Rollout drives the engine through its cursor/mount API.  Training sequences keep the
same structure for the prefix-tree trainer: the prefix is one unscored sequence, the
solver sequences share the planner's tokens as their prefix, and the verifier mounts
the prefix and the solvers' output ranges; every generated token is owned (trained)
by exactly one sequence.  Rewards are Bernoulli(p) per sample (synthetic), turned
into R = 2y - 1 and leave-one-out advantages over the instance's samples.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from ..rl.group import leave_one_out
from ..serving.engine import GenInput


@dataclass
class DagConfig:
    instances: int = 32
    samples: int = 4
    prefix_len: int = 2048
    turn_len: int = 512
    role_len: int = 16
    reward_p: float = 0.5
    temperature: float = 1.0
    seed: int = 0


@dataclass
class DagRollout:
    """Everything the trainer needs from one rollout of all instances."""

    flat: list = field(default_factory=list)       # per micro-unit (instance): list of token arrays
    mounts: list = field(default_factory=list)     # per instance: {seq index: [(at, src, s0, s1)]}
    loss_mask: list = field(default_factory=list)  # per instance: list of per-token masks
    behav: list = field(default_factory=list)      # per instance: list of per-token behaviour logprobs
    adv: list = field(default_factory=list)        # per instance: list of per-token advantages
    generated_tokens: int = 0
    rewards: list = field(default_factory=list)

    def microbatches(self, token_cap: int, build):
        return instance_microbatches(self, token_cap, build)


class MultiAgentDag:
    def __init__(self, vocab_size: int, cfg: DagConfig | None = None):
        self.cfg = cfg or DagConfig()
        self.vocab = vocab_size
        self.rng = np.random.default_rng(self.cfg.seed)
        self.step = 0

    def _tokens(self, n):
        return self.rng.integers(1, self.vocab, size=n, dtype=np.int64).astype(np.int32)

    def rollout(self, engine, instances: range | None = None) -> DagRollout:
        c = self.cfg
        inst = list(instances) if instances is not None else list(range(c.instances))
        self.step += 1
        tag = f"s{self.step}"
        prefixes = {i: self._tokens(c.prefix_len) for i in inst}
        roles = {name: self._tokens(c.role_len) for name in ("planner", "solver1", "solver2", "verifier")}
        # 1) prefill each instance's shared prefix (kept as a cursor; no generation)
        pre = engine.generate([GenInput(list(prefixes[i]), max_new_tokens=0, prefill_only=True,
                                        cursor_id=f"{tag}/p{i}", temperature=c.temperature) for i in inst])
        assert all(o.cursor for o in pre)
        S = c.samples
        keys = [(i, s) for i in inst for s in range(S)]
        # 2) planners: mount the prefix
        plan = engine.generate([GenInput(list(roles["planner"]), mount=[(f"{tag}/p{i}", 0, c.prefix_len)],
                                         max_new_tokens=c.turn_len, temperature=c.temperature,
                                         cursor_id=f"{tag}/pl{i}.{s}") for i, s in keys])
        # 3) solvers: continue (fork) the planner cursor
        sol_in = []
        for i, s in keys:
            for k in (1, 2):
                sol_in.append(GenInput(list(roles[f"solver{k}"]), cursor=f"{tag}/pl{i}.{s}",
                                       max_new_tokens=c.turn_len, temperature=c.temperature,
                                       cursor_id=f"{tag}/so{k}.{i}.{s}"))
        sol = engine.generate(sol_in)
        # 4) verifier: mount prefix + both solver outputs (rows with KV: all but the last token)
        ver_in = []
        for i, s in keys:
            m = [(f"{tag}/p{i}", 0, c.prefix_len)]
            for k in (1, 2):
                cur = engine.cursors.get(f"{tag}/so{k}.{i}.{s}")
                end = cur.length - 1
                m.append((cur.cid, end - (c.turn_len - 1), end))
            ver_in.append(GenInput(list(roles["verifier"]), mount=m, max_new_tokens=c.turn_len,
                                   temperature=c.temperature, cursor_id=f"{tag}/ve{i}.{s}"))
        ver = engine.generate(ver_in)

        out = DagRollout()
        out.generated_tokens = sum(len(o.output_ids) for o in plan + sol + ver)
        y = (self.rng.random(len(keys)) < c.reward_p).astype(np.float64)
        out.rewards = y.tolist()
        for ii, i in enumerate(inst):
            rs = [2.0 * y[ii * S + s] - 1.0 for s in range(S)]
            advs = leave_one_out(rs)
            seqs, masks, behs, advs_tok, mounts = [], [], [], [], {}
            seqs.append(prefixes[i].astype(np.int64))
            masks.append(np.zeros(c.prefix_len, np.float32))
            behs.append(np.zeros(c.prefix_len, np.float32))
            advs_tok.append(np.zeros(c.prefix_len, np.float32))
            for s in range(S):
                kidx = ii * S + s
                a = advs[s]
                p_out = plan[kidx]
                pl_tok = np.concatenate([roles["planner"], p_out.output_ids]).astype(np.int64)
                pl_mask = np.concatenate([np.zeros(c.role_len), np.ones(len(p_out.output_ids))]).astype(np.float32)
                pl_beh = np.concatenate([np.zeros(c.role_len), p_out.output_logprobs]).astype(np.float32)
                j_pl = len(seqs)
                seqs.append(pl_tok)
                masks.append(pl_mask)
                behs.append(pl_beh)
                advs_tok.append(np.full(len(pl_tok), a, np.float32))
                mounts[j_pl] = [(0, 0, 0, c.prefix_len)]
                sol_idx = []
                for k in (1, 2):
                    so = sol[kidx * 2 + (k - 1)]
                    tok = np.concatenate([pl_tok, roles[f"solver{k}"], so.output_ids]).astype(np.int64)
                    mask = np.concatenate([np.zeros(len(pl_tok) + c.role_len), np.ones(len(so.output_ids))])
                    beh = np.concatenate([np.zeros(len(pl_tok) + c.role_len), so.output_logprobs])
                    j = len(seqs)
                    seqs.append(tok)
                    masks.append(mask.astype(np.float32))
                    behs.append(beh.astype(np.float32))
                    advs_tok.append(np.full(len(tok), a, np.float32))
                    mounts[j] = [(0, 0, 0, c.prefix_len)]
                    sol_idx.append((j, len(tok)))
                vo = ver[kidx]
                vtok = np.concatenate([roles["verifier"], vo.output_ids]).astype(np.int64)
                j_v = len(seqs)
                seqs.append(vtok)
                masks.append(np.concatenate([np.zeros(c.role_len), np.ones(len(vo.output_ids))]).astype(np.float32))
                behs.append(np.concatenate([np.zeros(c.role_len), vo.output_logprobs]).astype(np.float32))
                advs_tok.append(np.full(len(vtok), a, np.float32))
                mounts[j_v] = [(0, 0, 0, c.prefix_len)] + [(0, j, n - c.turn_len, n - 1) for j, n in sol_idx]
            out.flat.append(seqs)
            out.mounts.append(mounts)
            out.loss_mask.append(masks)
            out.behav.append(behs)
            out.adv.append(advs_tok)
        # release this step's cursors (KV returns to the pool)
        for i, s in keys:
            for cid in (f"{tag}/pl{i}.{s}", f"{tag}/so1.{i}.{s}", f"{tag}/so2.{i}.{s}", f"{tag}/ve{i}.{s}"):
                engine.release_cursor(cid)
        for i in inst:
            engine.release_cursor(f"{tag}/p{i}")
        return out


def instance_microbatches(ro: DagRollout, token_cap: int, build):
    """Pack whole instances (mount units) into micro-batches of <= token_cap flat-unique tokens."""
    units = []
    for seqs, mounts, masks, behs, advs in zip(ro.flat, ro.mounts, ro.loss_mask, ro.behav, ro.adv):
        units.append((seqs, mounts, masks, behs, advs))
    groups, cur, cur_n = [], [], 0
    for u in units:
        # tree size of an instance: prefix + per sample (planner + 2 solver tails + verifier)
        n = sum(len(s) for s in u[0])
        est = len(u[0][0]) + sum(len(s) for s in u[0][1:]) // 2
        if cur and cur_n + est > token_cap:
            groups.append(cur)
            cur, cur_n = [], 0
        cur.append(u)
        cur_n += est
        del n
    if cur:
        groups.append(cur)
    mbs = []
    for g in groups:
        flat, cu, mounts, mask, beh, adv = [], [0], {}, [], [], []
        for seqs, m, masks, behs, advs in g:
            base = len(cu) - 1
            for j, s in enumerate(seqs):
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
