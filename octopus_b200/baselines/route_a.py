"""Route A: external ways of letting sibling B read sibling A, as conditions of the
cross-branch read probe (octopus_b200.tools.kv_read_probe), on this framework's engine.

Conditions: the probe's none / text / replay / K1 / K2 / K3, plus
  summary     A summarizes its context (greedy, at most --summary-tokens, decoded on A's own
              cache after a summary-request message); the summary goes into B's context
              after a header (Context-Folding / ReSum style summarize-then-read, zero-shot)
  kvcomm_sel  K3's relocated rows mounted on a layer subset only (KVComm-style selected-layer
              sharing; the subset is given by --mount-layers, not selected by a score)
With --mount-layers L, K1 / K2 / kvcomm_sel run on an engine that mounts only on layers L
(reported as `K1@L`, `K2@L`); K3 always mounts on every layer.  Without a subset kvcomm_sel
is K3 and is recorded `same_as` it.

    python -m octopus_b200.baselines.route_a run --probes probes.jsonl --out results.jsonl
        [--conditions none,text,summary,replay,K1,K2,K3,kvcomm_sel] [--mount-layers 8-15]
        [--preset qwen2.5-7b --layers 0 --checkpoint HF_DIR]
    python -m octopus_b200.baselines.route_a report results.jsonl [more.jsonl ...]

The report gives each condition's exact-match rate and paired differences with 95%
bootstrap intervals over probes (K1-K3, K2-K3, K1-K2, K2-summary, kvcomm_sel-K2,
kvcomm_sel-K3).  Probe files are kv_read_probe's (`build --synthetic N` makes one).

Reference parity (behaviour): `baselines/kv_read/route_a.py:1-45` (conditions summary and
kvcomm_sel on top of the KV-mount probe, mount on a layer subset, paired reports) and
`baselines/README.md` (condition definitions).
"""
from __future__ import annotations

import argparse
import json
import time

import numpy as np

from ..tools import kv_read_probe as kp

CONDITIONS = ("none", "text", "summary", "replay", "K1", "K2", "K3", "kvcomm_sel")
SUBSET = ("K1", "K2", "kvcomm_sel")  # the conditions --mount-layers applies to
PAIRS = (("K1", "K3"), ("K2", "K3"), ("K1", "K2"), ("K2", "summary"), ("kvcomm_sel", "K2"), ("kvcomm_sel", "K3"))


def parse_layers(spec: str, n_layers: int) -> list[int] | None:
    """--mount-layers: all, a-b (inclusive) or i,j,..."""
    if not spec or spec == "all":
        return None
    a, _, b = spec.partition("-")
    out = list(range(int(a), int(b) + 1)) if b else sorted({int(x) for x in spec.split(",")})
    if not out or min(out) < 0 or max(out) >= n_layers:
        raise ValueError(f"mount layers {spec!r} outside 0..{n_layers - 1}")
    return out


def summary_condition(engine, p: dict, request: list, summary_tokens: int, tag: str, temperature: float = 1e-3):
    """B's answer after reading A's summary; returns (result, summary record)."""
    from ..serving.engine import GenInput

    a_cur = f"{tag}/Asum"
    t0 = time.perf_counter()
    engine.generate([GenInput(list(p["a_prefix"]) + list(p["a_turns"]), max_new_tokens=0, prefill_only=True,
                              cursor_id=a_cur, temperature=temperature)])
    s = engine.generate([GenInput(list(request), cursor=a_cur, max_new_tokens=summary_tokens, keep_cursor=False,
                                  temperature=temperature)])[0].output_ids
    engine.release_cursor(a_cur)
    ms = (time.perf_counter() - t0) * 1e3
    q = dict(p, b_prefix=list(p["b_prefix"]) + list(p.get("header", [])) + list(s))
    r = kp.run_probe(engine, q, ("none",), tag=f"{tag}/sum", temperature=temperature)["none"]
    return r, {"summary_tokens": len(s), "summary_ms": round(ms, 2)}


def run_one(engine, sub_engine, p: dict, conditions, tag: str, request: list, summary_tokens: int,
            temperature: float = 1e-3) -> dict:
    res = {}
    base = [c for c in conditions if c in kp.CONDITIONS and not (sub_engine is not None and c in SUBSET)]
    if base:
        res.update(kp.run_probe(engine, p, base, tag=f"{tag}/all", temperature=temperature))
    if sub_engine is not None:
        sub = [c for c in conditions if c in SUBSET]
        mapped = ["K3" if c == "kvcomm_sel" else c for c in sub]
        if mapped:
            got = kp.run_probe(sub_engine, p, tuple(dict.fromkeys(mapped)), tag=f"{tag}/sub", temperature=temperature)
            for c, m in zip(sub, mapped):
                res[c] = dict(got[m], layers="subset")
    elif "kvcomm_sel" in conditions:
        if "K3" not in res:
            res["K3"] = kp.run_probe(engine, p, ("K3",), tag=f"{tag}/k3", temperature=temperature)["K3"]
        res["kvcomm_sel"] = dict(res["K3"], same_as="K3")
    if "summary" in conditions:
        r, rec = summary_condition(engine, p, request, summary_tokens, tag, temperature)
        res["summary"] = dict(r, **rec)
    return res


def _boot(diff: np.ndarray, n: int = 2000, seed: int = 0) -> tuple[float, float]:
    rng = np.random.default_rng(seed)
    idx = rng.integers(0, len(diff), (n, len(diff)))
    m = diff[idx].mean(axis=1)
    return float(np.percentile(m, 2.5)), float(np.percentile(m, 97.5))


def report(rows: list[dict]) -> dict:
    out = {"conditions": {}, "pairs": {}}
    for c in CONDITIONS:
        v = [r["conditions"][c] for r in rows if c in r.get("conditions", {})]
        if v:
            out["conditions"][c] = {"n": len(v), "exact": float(np.mean([x["exact"] for x in v])),
                                    "prefix": float(np.mean([x["prefix"] for x in v]))}
    for a, b in PAIRS:
        both = [r["conditions"] for r in rows if a in r.get("conditions", {}) and b in r.get("conditions", {})]
        if both:
            d = np.asarray([float(x[a]["exact"]) - float(x[b]["exact"]) for x in both])
            lo, hi = _boot(d)
            out["pairs"][f"{a} - {b}"] = {"n": len(d), "mean": float(d.mean()), "ci95": [lo, hi]}
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m octopus_b200.baselines.route_a")
    sub = ap.add_subparsers(dest="cmd", required=True)
    r = sub.add_parser("run")
    r.add_argument("--probes", required=True)
    r.add_argument("--out", required=True)
    r.add_argument("--conditions", default=",".join(CONDITIONS))
    r.add_argument("--mount-layers", default="all")
    r.add_argument("--summary-tokens", type=int, default=192)
    r.add_argument("--preset", default="qwen2.5-7b")
    r.add_argument("--layers", type=int, default=0)
    r.add_argument("--checkpoint", default="")
    r.add_argument("--kv-slots", type=int, default=1 << 20)
    rp = sub.add_parser("report")
    rp.add_argument("results", nargs="+")
    args = ap.parse_args(argv)
    if args.cmd == "report":
        rows = []
        for fn in args.results:
            with open(fn) as f:
                rows += [json.loads(x) for x in f if x.strip()]
        print(json.dumps(report(rows), indent=1))
        return 0
    import torch

    from ..models.config import get_config
    from ..models.decoder import FlatLayout, Weights, init_flat, load_hf
    from ..serving.engine import Engine

    dev = torch.device("cuda", 0) if torch.cuda.is_available() else torch.device("cpu")
    cfg = get_config(args.preset, layers=args.layers) if args.layers else get_config(args.preset)
    lay = FlatLayout(cfg)
    w = Weights(cfg, init_flat(cfg, lay, dev, seed=0), lay)
    if args.checkpoint:
        load_hf(w, args.checkpoint)
    layers = parse_layers(args.mount_layers, cfg.layers)
    eng = Engine(cfg, w, kv_slots=args.kv_slots, max_batch=8, device=dev)
    sub_eng = Engine(cfg, w, kv_slots=args.kv_slots, max_batch=8, device=dev, mount_layers=layers) if layers else None
    conds = [c for c in args.conditions.split(",") if c]
    request = list(np.random.default_rng(7).integers(1, cfg.vocab_size, 24))  # the summary request (token ids)
    rows = []
    with open(args.probes) as f, open(args.out, "w") as g:
        for i, line in enumerate(f):
            if not line.strip():
                continue
            res = run_one(eng, sub_eng, json.loads(line), conds, f"p{i}", request, args.summary_tokens)
            rows.append({"probe": i, "mount_layers": args.mount_layers, "conditions": res})
            g.write(json.dumps(rows[-1], default=int) + "\n")
    print(json.dumps(report(rows)))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
