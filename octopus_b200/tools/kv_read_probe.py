"""Cross-branch KV read probe: can thread B use sibling A's turns when they are mounted into
B's context as A computed them, and under which position rule?

Conditions at each probe (A's turns = the rows of A's context after its prefix):
  none    B alone
  text    A's turns as tokens in B's context after a short header (every layer recomputes
          them from B's state)
  replay  A's turn tokens spliced into B's context (recomputed, no header)
  K1      A's turn rows mounted at their original positions; B continues at its own next
  K2      mounted; B continues at max(its next position, last mounted position + 1)
  K3      mounted, relocated to B's next positions (keys re-rotated by the offset); B
          continues after them
Each condition asks B the probe's question (a cue from A's turns) and decodes greedily
(temperature 1e-3); the score is the fraction of the answer's leading tokens reproduced
(`prefix`) and whether all were (`exact`).

Probe file (JSONL, token ids): {"a_prefix": [...], "a_turns": [...], "b_prefix": [...],
"question": [...], "answer": [...], "header": [...] (optional, for `text`)}.

    python -m octopus_b200.tools.kv_read_probe build --synthetic 32 --out probes.jsonl [--vocab 152064]
    python -m octopus_b200.tools.kv_read_probe run --probes probes.jsonl --out results.jsonl
        [--preset qwen2.5-7b --layers 0 --checkpoint HF_DIR] [--conditions none text replay K1 K2 K3]
    python -m octopus_b200.tools.kv_read_probe report results.jsonl

Synthetic probes plant a fact (cue tokens followed by answer tokens) in A's turns and ask
B to continue the cue: random-init weights give chance-level scores; a trained checkpoint
(--checkpoint, Hugging Face safetensors) gives the measurement.

Reference parity (behaviour): `octopus/tools/kv_read_probe.py:1-17` (conditions none, text,
replay, K1, K2, K3; build / run / report).  K1 and K3 are the engine's `mount_rule`
(serving/engine.py); the trainer's prefix tree reproduces K2.
"""
from __future__ import annotations

import argparse
import json

import numpy as np

CONDITIONS = ("none", "text", "replay", "K1", "K2", "K3")


def synthetic_probes(n: int, vocab: int, seed: int = 0, a_len: int = 256, turn_len: int = 128, b_len: int = 256,
                     cue_len: int = 8, answer_len: int = 4) -> list[dict]:
    rng = np.random.default_rng(seed)
    tok = lambda k: rng.integers(1, vocab, k).tolist()  # noqa: E731
    out = []
    for _ in range(n):
        cue, ans = tok(cue_len), tok(answer_len)
        turns = tok(turn_len)
        at = int(rng.integers(0, turn_len - cue_len - answer_len))
        turns[at:at + cue_len + answer_len] = cue + ans
        out.append({"a_prefix": tok(a_len), "a_turns": turns, "b_prefix": tok(b_len), "question": cue,
                    "answer": ans, "header": tok(6)})
    return out


def run_probe(engine, p: dict, conditions=CONDITIONS, tag: str = "p", temperature: float = 1e-3) -> dict:
    """Scores of one probe under each condition."""
    from ..serving.engine import GenInput

    ans = list(p["answer"])
    n = len(ans)
    res = {}
    a_cur, b_cur = f"{tag}/A", f"{tag}/B"
    mounted = any(c in ("K1", "K2", "K3") for c in conditions)
    if mounted:
        engine.generate([GenInput(list(p["a_prefix"]) + list(p["a_turns"]), max_new_tokens=0, prefill_only=True,
                                  cursor_id=a_cur, temperature=temperature),
                         GenInput(list(p["b_prefix"]), max_new_tokens=0, prefill_only=True, cursor_id=b_cur,
                                  temperature=temperature)])
    la, lt = len(p["a_prefix"]), len(p["a_turns"])
    for c in conditions:
        if c == "none":
            g = GenInput(list(p["b_prefix"]) + list(p["question"]), max_new_tokens=n)
        elif c == "text":
            g = GenInput(list(p["b_prefix"]) + list(p.get("header", [])) + list(p["a_turns"]) + list(p["question"]),
                         max_new_tokens=n)
        elif c == "replay":
            g = GenInput(list(p["b_prefix"]) + list(p["a_turns"]) + list(p["question"]), max_new_tokens=n)
        elif c in ("K1", "K2", "K3"):
            g = GenInput(list(p["question"]), cursor=b_cur, mount=[(a_cur, la, la + lt)], mount_rule=c,
                         max_new_tokens=n)
        else:
            raise ValueError(f"unknown condition {c!r}")
        g.temperature, g.keep_cursor = temperature, False
        o = engine.generate([g])[0]
        k = 0
        while k < n and k < len(o.output_ids) and o.output_ids[k] == ans[k]:
            k += 1
        res[c] = {"prefix": k / n if n else 1.0, "exact": k == n, "logprob": float(np.sum(o.output_logprobs)),
                  "first_pos": o.first_pos, "output": o.output_ids}
    if mounted:
        engine.release_cursor(a_cur)
        engine.release_cursor(b_cur)
    return res


def report(rows: list[dict]) -> dict:
    out = {}
    for c in CONDITIONS:
        vals = [r["conditions"][c] for r in rows if c in r.get("conditions", {})]
        if vals:
            out[c] = {"n": len(vals), "prefix": float(np.mean([v["prefix"] for v in vals])),
                      "exact": float(np.mean([v["exact"] for v in vals]))}
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m octopus_b200.tools.kv_read_probe")
    sub = ap.add_subparsers(dest="cmd", required=True)
    b = sub.add_parser("build")
    b.add_argument("--synthetic", type=int, default=32)
    b.add_argument("--vocab", type=int, default=152064)
    b.add_argument("--seed", type=int, default=0)
    b.add_argument("--out", required=True)
    r = sub.add_parser("run")
    r.add_argument("--probes", required=True)
    r.add_argument("--out", required=True)
    r.add_argument("--preset", default="qwen2.5-7b")
    r.add_argument("--layers", type=int, default=0)
    r.add_argument("--checkpoint", default="")
    r.add_argument("--conditions", nargs="+", default=list(CONDITIONS))
    r.add_argument("--kv-slots", type=int, default=1 << 20)
    rp = sub.add_parser("report")
    rp.add_argument("results")
    args = ap.parse_args(argv)
    if args.cmd == "build":
        with open(args.out, "w") as f:
            for p in synthetic_probes(args.synthetic, args.vocab, args.seed):
                f.write(json.dumps(p) + "\n")
        return 0
    if args.cmd == "report":
        with open(args.results) as f:
            print(json.dumps(report([json.loads(x) for x in f if x.strip()]), indent=1))
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
    eng = Engine(cfg, w, kv_slots=args.kv_slots, max_batch=8, device=dev)
    with open(args.probes) as f, open(args.out, "w") as g:
        rows = []
        for i, line in enumerate(f):
            if not line.strip():
                continue
            res = run_probe(eng, json.loads(line), args.conditions, tag=f"p{i}")
            rows.append({"probe": i, "conditions": res})
            g.write(json.dumps(rows[-1]) + "\n")
    print(json.dumps(report(rows)))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
