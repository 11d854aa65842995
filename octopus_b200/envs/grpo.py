"""Synthetic single-agent GRPO environment: prompts of uniform random
tokens, `samples` responses per prompt sampled at the configured temperature up to
`response_len` tokens, Bernoulli(p) rewards, R = 2y - 1 and leave-one-out advantages over
each prompt's samples.

The samples of a prompt share it as a prefix: the trainer's prefix tree stores the
prompt once per micro-batch and trains every response token once.  Micro-batches hold
whole prompt groups up to a token cap (tree tokens: prompt + its responses).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from ..rl.group import leave_one_out
from ..serving.engine import GenInput


@dataclass
class GrpoConfig:
    prompts: int = 64
    samples: int = 8
    prompt_len: int = 512
    response_len: int = 1024
    reward_p: float = 0.5
    temperature: float = 1.0
    seed: int = 0


@dataclass
class GrpoRollout:
    groups: list = field(default_factory=list)  # per prompt: (seqs, masks, behs, advs)
    generated_tokens: int = 0
    rewards: list = field(default_factory=list)

    def microbatches(self, token_cap: int, build):
        out, cur, cur_n = [], [], 0
        for g in self.groups:
            seqs = g[0]
            n = len(seqs[0]) + sum(len(s) for s in seqs) - len(seqs) * self._prompt(seqs)
            if cur and cur_n + n > token_cap:
                out.append(cur)
                cur, cur_n = [], 0
            cur.append(g)
            cur_n += n
        if cur:
            out.append(cur)
        mbs = []
        for part in out:
            flat, cu, mask, beh, adv = [], [0], [], [], []
            for seqs, masks, behs, advs in part:
                for s, m, b, a in zip(seqs, masks, behs, advs):
                    flat.append(s)
                    cu.append(cu[-1] + len(s))
                    mask.append(m)
                    beh.append(b)
                    adv.append(a)
            mbs.append(build(np.concatenate(flat), cu, None, np.concatenate(mask), np.concatenate(adv),
                             np.concatenate(beh)))
        return mbs

    @staticmethod
    def _prompt(seqs) -> int:
        a = seqs[0]
        n = len(a)
        for s in seqs[1:]:
            m = min(n, len(s))
            neq = np.nonzero(a[:m] != s[:m])[0]
            n = int(neq[0]) if len(neq) else m
        return n


class SingleAgentGrpo:
    def __init__(self, vocab_size: int, cfg: GrpoConfig | None = None):
        self.cfg = cfg or GrpoConfig()
        self.vocab = vocab_size
        self.rng = np.random.default_rng(self.cfg.seed)
        self.step = 0

    def rollout(self, engine, prompts=None) -> GrpoRollout:
        c = self.cfg
        idx = list(prompts) if prompts is not None else list(range(c.prompts))
        self.step += 1
        toks = {i: self.rng.integers(1, self.vocab, c.prompt_len).astype(np.int64) for i in idx}
        # each prompt is prefilled once (all but its last token, kept as a cursor); its samples
        # continue that cursor from the last prompt token, sharing the prompt's KV
        tag = f"g{self.step}"
        engine.generate([GenInput(toks[i][:-1].tolist(), max_new_tokens=0, prefill_only=True,
                                  cursor_id=f"{tag}/p{i}", temperature=c.temperature) for i in idx])
        reqs = [GenInput([int(toks[i][-1])], cursor=f"{tag}/p{i}", max_new_tokens=c.response_len,
                         temperature=c.temperature, keep_cursor=False) for i in idx for _ in range(c.samples)]
        outs = engine.generate(reqs)
        for i in idx:
            engine.release_cursor(f"{tag}/p{i}")
        ro = GrpoRollout()
        ro.generated_tokens = sum(len(o.output_ids) for o in outs)
        y = (self.rng.random(len(outs)) < c.reward_p).astype(np.float64)
        ro.rewards = y.tolist()
        for k, i in enumerate(idx):
            group = outs[k * c.samples:(k + 1) * c.samples]
            advs = leave_one_out([2.0 * y[k * c.samples + s] - 1.0 for s in range(c.samples)])
            seqs, masks, behs, adv = [], [], [], []
            for o, a in zip(group, advs):
                n = len(o.output_ids)
                seqs.append(np.concatenate([toks[i], np.asarray(o.output_ids, np.int64)]))
                masks.append(np.concatenate([np.zeros(c.prompt_len), np.ones(n)]).astype(np.float32))
                behs.append(np.concatenate([np.zeros(c.prompt_len), o.output_logprobs]).astype(np.float32))
                adv.append(np.full(c.prompt_len + n, a, np.float32))
            ro.groups.append((seqs, masks, behs, adv))
        return ro
