"""Per-request prompt cost at L tokens of history: re-rendering the whole conversation vs
rendering only the new messages after the cursor (render_delta).

    python -m octopus_b200.tools.delta_render_bench [--tokens 8000 32000 128000] [--tokenizer HF_DIR]

The history repeats a fixed tool-calling exchange until it holds about L tokens; the
request is one turn of tool results.  Reports milliseconds per request for both paths.

Reference parity (behaviour): `octopus/tools/delta_render_bench.py` (the cursor protocol's
prompt-assembly numbers in docs/cursor-protocol.md).
"""
from __future__ import annotations

import argparse
import json
import time


def conversation(n_turns: int):
    call = {"id": "c1", "type": "function", "function": {"name": "shell", "arguments": '{"cmd": "pytest -x"}'}}
    msgs = [{"role": "system", "content": "You fix bugs in a repository."},
            {"role": "user", "content": "Fix the failing test in module parser."}]
    for i in range(n_turns):
        msgs.append({"role": "assistant", "content": f"Step {i}: running the tests again.", "tool_calls": [call]})
        msgs.append({"role": "tool", "tool_call_id": "c1",
                     "content": "FAILED tests/test_parser.py::test_case_%d - AssertionError: expected 3 got 4 " % i
                     * 4})
    return msgs


def bench(tok, target_tokens: int, reps: int = 5) -> dict:
    per_turn = len(tok.apply(conversation(1), None, False)) - len(tok.apply(conversation(0), None, False))
    n = max(1, target_tokens // max(1, per_turn))
    hist = conversation(n)
    new = [{"role": "tool", "tool_call_id": "c1", "content": "1 passed in 0.2s"}]
    t0 = time.perf_counter()
    for _ in range(reps):
        tok.apply(hist + new, None, True)
    full = (time.perf_counter() - t0) / reps
    t0 = time.perf_counter()
    for _ in range(reps):
        tok.render_delta(new)
    delta = (time.perf_counter() - t0) / reps
    return {"history_tokens": len(tok.apply(hist, None, False)), "full_ms": round(full * 1e3, 3),
            "delta_ms": round(delta * 1e3, 3), "speedup": round(full / max(delta, 1e-9), 1)}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m octopus_b200.tools.delta_render_bench")
    ap.add_argument("--tokens", type=int, nargs="*", default=[8000, 32000, 128000])
    ap.add_argument("--tokenizer", default="")
    args = ap.parse_args(argv)
    from ..serving.chat import ChatTokenizer

    tok = ChatTokenizer.from_dir(args.tokenizer) if args.tokenizer else ChatTokenizer.tiny()
    for L in args.tokens:
        print(json.dumps(bench(tok, L)))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
