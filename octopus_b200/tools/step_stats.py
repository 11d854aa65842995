"""Per-step training stats of a run: reward, entropy, grad norm, clip ratio, tokens, time.

    python -m octopus_b200.tools.step_stats RUN_DIR/steps.jsonl

Reads the trainer's step lines (python -m octopus_b200.rl.train writes one JSON object per
step) and prints a table; missing keys show as '-'.

Reference parity (behaviour): `octopus/tools/step_stats.py` (task reward, entropy, grad
norm, clip ratio, train/infer logprob gap per step of a trial's log).
"""
from __future__ import annotations

import json
import sys

KEYS = [("mean_reward", "reward"), ("entropy", "entropy"), ("grad_norm", "grad_norm"), ("clip_frac", "clip"),
        ("logp_diff", "logp_gap"), ("generated_tokens", "tokens"), ("time", "time_s")]


def table(rows: list[dict]) -> str:
    out = ["step | " + " | ".join(h for _, h in KEYS)]
    for r in rows:
        vals = []
        for k, _ in KEYS:
            v = r.get(k)
            vals.append("-" if v is None else (f"{v:.4g}" if isinstance(v, float) else str(v)))
        out.append(f"{r.get('step', '?')} | " + " | ".join(vals))
    return "\n".join(out)


def main(argv=None) -> int:
    argv = sys.argv[1:] if argv is None else argv
    if len(argv) != 1:
        print(__doc__)
        return 2
    rows = [json.loads(x) for x in open(argv[0]) if x.strip().startswith("{")]
    print(table(rows))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
