"""GRPO / decoupled-PPO policy loss over scored (row, label) pairs.

Per token: ratio r = exp(logp - prox) with prox the proximal policy's logprob (with
``reuse_train_logp`` prox = the detached train logprob, so r == 1 but its gradient is
A * d logp), clipped PPO objective with separate low/high clip (clip-higher), and the
decoupled behaviour weight w = exp(prox - behaviour) of the rollout policy; tokens
with w above ``behav_imp_weight_cap`` are rejected (rejection sampling).  The loss is a
token-mean over the whole step (denominator = every loss-mask token of the step, on
every rank), so micro-batch splits do not change it.

Reference parity: `octopus/rl/grpo.yaml:103-123` (decoupled PPO: eps_clip 0.2,
eps_clip_higher 0.28, behav_imp_weight_cap 5, reuse_train_logp, adv_norm mean-only at
group level) and AReaL's grpo_loss_fn semantics it configures.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class PPOConfig:
    eps_clip: float = 0.2
    eps_clip_higher: float | None = 0.28
    behav_imp_weight_cap: float | None = 5.0
    reuse_train_logp: bool = True
    entropy_coef: float = 0.0
    kl_coef: float = 0.0


def ppo_loss(logp: torch.Tensor, ent: torch.Tensor, adv: torch.Tensor, weight: torch.Tensor,
             behav_logp: torch.Tensor | None, prox_logp: torch.Tensor | None, denom: float, cfg: PPOConfig):
    """Returns (loss scalar, stats dict of detached tensors).

    logp, ent: [P] (differentiable); adv, weight (loss-mask count per pair), behav_logp,
    prox_logp: [P]; denom: total loss-mask tokens of the whole step.
    """
    prox = logp.detach() if (cfg.reuse_train_logp or prox_logp is None) else prox_logp.float()
    ratio = torch.exp(logp - prox)
    lo = 1.0 - cfg.eps_clip
    hi = 1.0 + (cfg.eps_clip_higher if cfg.eps_clip_higher is not None else cfg.eps_clip)
    clipped = ratio.clamp(lo, hi)
    pg = -torch.minimum(ratio * adv, clipped * adv)
    w = weight.float()
    if behav_logp is not None:
        bw = torch.exp(prox - behav_logp.float())
        if cfg.behav_imp_weight_cap is not None:
            keep = (bw <= cfg.behav_imp_weight_cap).float()
            w = w * keep
        pg = pg * bw
    loss = (pg * w).sum()
    if cfg.entropy_coef:
        loss = loss - cfg.entropy_coef * (ent * w).sum()
    if cfg.kl_coef and behav_logp is not None:
        loss = loss + cfg.kl_coef * ((logp - behav_logp.float()) * w).sum()
    loss = loss / max(float(denom), 1.0)
    with torch.no_grad():
        n = w.sum().clamp(min=1.0)
        stats = {
            "clip_frac": (((ratio < lo) | (ratio > hi)).float() * w).sum() / n,
            "entropy": (ent.detach() * w).sum() / n,
            "logp": (logp.detach() * w).sum() / n,
            "behave_approx_kl": (((behav_logp.float() - prox) if behav_logp is not None else torch.zeros_like(prox))
                                 * w).sum() / n,
            "tokens": w.sum(),
        }
    return loss, stats
