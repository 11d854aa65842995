"""Cluster bootstrap intervals for grouped binary / real outcomes.

Samples of one question (all runs of one task) are not independent, so intervals
resample whole clusters.  One resampling is drawn as multinomial cluster weights
(how often each cluster is picked in a bootstrap replicate), so every statistic is a
ratio of weighted cluster sums: a pooled mean is (W @ sums) / (W @ counts), a contrast
between two arms is the difference of two such ratios.  Intervals are the 2.5 / 97.5
percentiles over replicates; estimates are the plain pooled values.
"""
from __future__ import annotations

import numpy as np

NAN3 = (float("nan"), float("nan"), float("nan"))


def _weights(n_clusters: int, reps: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return rng.multinomial(n_clusters, np.full(n_clusters, 1.0 / n_clusters), size=reps).astype(np.float64)


def pooled_ci(groups: list[list[float]], reps: int = 2000, seed: int = 0) -> tuple[float, float, float]:
    """(pooled mean, lo, hi) of grouped values; empty groups are ignored."""
    groups = [g for g in groups if len(g)]
    if not groups:
        return NAN3
    sums = np.array([float(sum(g)) for g in groups])
    counts = np.array([float(len(g)) for g in groups])
    w = _weights(len(groups), reps, seed)
    est = (w @ sums) / (w @ counts)
    return float(sums.sum() / counts.sum()), float(np.percentile(est, 2.5)), float(np.percentile(est, 97.5))


def contrast_ci(rows: list[dict], value, in_arm, reps: int = 2000, seed: int = 0) -> tuple[float, float, float]:
    """(mean of value over rows in the arm - mean over the others, lo, hi), clusters
    resampled whole (rows carry a "cluster" key).  NaN when an arm is empty."""
    table: dict = {}
    for row in rows:
        acc = table.setdefault(row["cluster"], np.zeros(4))
        v = float(value(row))
        if in_arm(row):
            acc[0] += v
            acc[1] += 1
        else:
            acc[2] += v
            acc[3] += 1
    if not table:
        return NAN3
    s = np.stack(list(table.values()))
    tot = s.sum(0)
    if tot[1] == 0 or tot[3] == 0:
        return NAN3
    w = _weights(len(s), reps, seed)
    ws = w @ s
    with np.errstate(invalid="ignore", divide="ignore"):
        est = ws[:, 0] / ws[:, 1] - ws[:, 2] / ws[:, 3]
    point = tot[0] / tot[1] - tot[2] / tot[3]
    return float(point), float(np.nanpercentile(est, 2.5)), float(np.nanpercentile(est, 97.5))


def by_cluster(rows: list[dict], value) -> list[list[float]]:
    groups: dict = {}
    for row in rows:
        groups.setdefault(row["cluster"], []).append(float(value(row)))
    return list(groups.values())


def ci_text(ci) -> str:
    return f"{ci[0]:.3f} [{ci[1]:.3f}, {ci[2]:.3f}]"
