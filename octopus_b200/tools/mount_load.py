"""Mount load: forced cross-thread reads (cursor + mount requests) on the engine.

PAIRS thread pairs run at a time, replaced as they finish, until DURATION seconds passed or
every pair is done.  A pair is a fork: a root request of ROOT tokens, then two sibling threads
continuing from the root's reply, each taking TURNS turns (a tool result of lognormal size,
median TOOL tokens, sent from the thread's last cursor, then a sampled reply of REPLY tokens).
Every 2-5 turns thread 0 reads its sibling (thread 1 reads every 6-10 turns, so it stays a
long source): the read turn carries a short tool result and mounts the end of the sibling's
own tokens before its last reply (never its fork prefix, never rows it mounted itself), M
tokens with M lognormal (median MOUNT), capped by what the sibling has.  Later turns of the
reader continue from cursors that hold the mounted rows.  A request whose cursor is gone
(404: evicted) ends its thread.  One JSON line per request; a summary line.

    python -m octopus_b200.tools.mount_load --pairs 8 --duration 120 [--turns 15 30] [--root 8000]
        [--tool 500] [--reply 40 500] [--mount 949] [--preset qwen2.5-7b --layers 0] [--out reqs.jsonl]

The turns of all live threads go to the engine as one batch per round (the engine batches
requests; a round is the concurrency of PAIRS pairs).

Reference parity (behaviour): `octopus/tools/mount_load.py:1-17` (fork pairs, sibling turns,
forced reads mounting the end of the sibling's own tokens, lognormal sizes, per-request
records).
"""
from __future__ import annotations

import argparse
import json
import math
import time
from dataclasses import dataclass, field

import numpy as np


@dataclass
class _Thread:
    pair: int
    idx: int
    cursor: str
    fork_len: int                 # rows of the shared fork prefix (root prompt + reply)
    turns_left: int
    next_read: int
    turn: int = 0
    last_reply_start: int = 0     # cursor row where the last reply began
    alive: bool = True
    log: list = field(default_factory=list)


def _lognormal(rng, median: float, sigma: float = 1.0, lo: int = 1, hi: int = 1 << 30) -> int:
    return int(min(hi, max(lo, round(median * math.exp(sigma * rng.standard_normal())))))


def _mount_range(cur, fork_len: int, end: int, want: int):
    """[a, b): the last rows before `end` of the cursor's own (not fork, not mounted) tokens,
    at most `want` of them."""
    own = ~cur.mounted[:end]
    own[:fork_len] = False
    b = end
    while b > fork_len and not own[b - 1]:
        b -= 1
    a = b
    while a > fork_len and own[a - 1] and b - a < want:
        a -= 1
    return (a, b) if b > a else None


def run(engine, vocab: int, pairs: int, duration: float, n_pairs_total: int | None = None, turns=(15, 30),
        root: int = 8000, tool: int = 500, reply=(40, 500), mount: int = 949, seed: int = 0, out=None) -> dict:
    from ..serving.engine import CursorNotFound, GenInput

    rng = np.random.default_rng(seed)
    tok = lambda n: rng.integers(1, vocab, n).tolist()  # noqa: E731
    t_start = time.perf_counter()
    n_pairs_total = n_pairs_total if n_pairs_total is not None else pairs
    started, threads = 0, []
    stats = {"requests": 0, "reads": 0, "mounted_tokens": 0, "not_found": 0, "prompt_tokens": 0,
             "cached_tokens": 0, "generated_tokens": 0}

    def log(row):
        stats["requests"] += 1
        if out is not None:
            out.write(json.dumps(row) + "\n")

    def start_pair(p):
        rid = f"ml{seed}-{p}"
        t0 = time.perf_counter()
        o = engine.generate([GenInput(tok(root), max_new_tokens=int(rng.integers(*reply)), cursor_id=f"{rid}/root")])[0]
        log({"pair": p, "thread": -1, "turn": 0, "kind": "root", "seconds": round(time.perf_counter() - t0, 4),
             "prompt_tokens": o.prompt_tokens, "cached_tokens": o.cached_tokens, "generated": len(o.output_ids)})
        stats["prompt_tokens"] += o.prompt_tokens
        stats["generated_tokens"] += len(o.output_ids)
        fork = engine.cursors.get(o.cursor).length
        return [_Thread(p, i, o.cursor, fork, int(rng.integers(*turns)),
                        int(rng.integers(2, 6)) if i == 0 else int(rng.integers(6, 11))) for i in range(2)]

    while (started < n_pairs_total or threads) and time.perf_counter() - t_start < duration:
        while started < n_pairs_total and len({t.pair for t in threads}) < pairs:
            threads += start_pair(started)
            started += 1
        batch, meta = [], []
        reply_start = {id(t): t.last_reply_start for t in threads}  # the round's snapshot (cursors not yet advanced)
        for th in threads:
            th.turn += 1
            sib = next((s for s in threads if s.pair == th.pair and s.idx != th.idx), None)
            mounts, kind = [], "turn"
            if sib is not None and th.turn == th.next_read:
                sc = engine.cursors.get(sib.cursor)
                end = min(sc.length, reply_start[id(sib)] or sc.length) if sc is not None else 0
                rng_ = _mount_range(sc, sib.fork_len, end, _lognormal(rng, mount)) if sc is not None else None
                if rng_ is not None:
                    mounts, kind = [(sib.cursor, rng_[0], rng_[1])], "read"
                th.next_read += int(rng.integers(2, 6)) if th.idx == 0 else int(rng.integers(6, 11))
            n_tool = 60 if kind == "read" else _lognormal(rng, tool)
            cur = engine.cursors.get(th.cursor)
            th.last_reply_start = (cur.length if cur is not None else 0) + n_tool + sum(b - a for _, a, b in mounts)
            batch.append(GenInput(tok(n_tool), cursor=th.cursor, mount=mounts, max_new_tokens=int(rng.integers(*reply)),
                                  cursor_id=f"{th.cursor.split('/')[0]}/t{th.idx}.{th.turn}"))
            meta.append((th, kind, sum(b - a for _, a, b in mounts)))
        if not batch:
            break
        t0 = time.perf_counter()
        try:
            outs = engine.generate(batch)
        except CursorNotFound:
            outs = []
            for g in batch:  # find the thread(s) whose cursor is gone, keep the others
                try:
                    outs.append(engine.generate([g])[0])
                except CursorNotFound:
                    outs.append(None)
        dt = time.perf_counter() - t0
        for (th, kind, m), o in zip(meta, outs):
            if o is None:
                stats["not_found"] += 1
                th.alive = False
                log({"pair": th.pair, "thread": th.idx, "turn": th.turn, "kind": kind, "status": 404})
                continue
            th.cursor = o.cursor
            th.turns_left -= 1
            stats["reads"] += kind == "read"
            stats["mounted_tokens"] += m
            stats["prompt_tokens"] += o.prompt_tokens
            stats["cached_tokens"] += o.cached_tokens
            stats["generated_tokens"] += len(o.output_ids)
            log({"pair": th.pair, "thread": th.idx, "turn": th.turn, "kind": kind, "mounted": m,
                 "batch_seconds": round(dt, 4), "prompt_tokens": o.prompt_tokens, "cached_tokens": o.cached_tokens,
                 "generated": len(o.output_ids)})
            if th.turns_left <= 0:
                th.alive = False
        threads = [t for t in threads if t.alive]
    wall = time.perf_counter() - t_start
    stats.update({"pairs": started, "seconds": round(wall, 3),
                  "generated_tokens_per_s": round(stats["generated_tokens"] / wall, 2) if wall > 0 else None})
    return stats


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m octopus_b200.tools.mount_load")
    ap.add_argument("--pairs", type=int, default=8)
    ap.add_argument("--total", type=int, default=0, help="pairs to run in all (0: --pairs)")
    ap.add_argument("--duration", type=float, default=120.0)
    ap.add_argument("--turns", type=int, nargs=2, default=[15, 30])
    ap.add_argument("--root", type=int, default=8000)
    ap.add_argument("--tool", type=int, default=500)
    ap.add_argument("--reply", type=int, nargs=2, default=[40, 500])
    ap.add_argument("--mount", type=int, default=949)
    ap.add_argument("--preset", default="qwen2.5-7b")
    ap.add_argument("--layers", type=int, default=0)
    ap.add_argument("--kv-slots", type=int, default=1 << 21)
    ap.add_argument("--out", default="")
    args = ap.parse_args(argv)

    import torch

    from ..models.config import get_config
    from ..models.decoder import FlatLayout, Weights, init_flat
    from ..serving.engine import Engine

    dev = torch.device("cuda", 0) if torch.cuda.is_available() else torch.device("cpu")
    cfg = get_config(args.preset, layers=args.layers) if args.layers else get_config(args.preset)
    lay = FlatLayout(cfg)
    eng = Engine(cfg, Weights(cfg, init_flat(cfg, lay, dev, seed=0), lay), kv_slots=args.kv_slots,
                 max_batch=max(8, 2 * args.pairs), device=dev)
    f = open(args.out, "w") if args.out else None
    try:
        summary = run(eng, cfg.vocab_size, args.pairs, args.duration, args.total or args.pairs, tuple(args.turns),
                      args.root, args.tool, tuple(args.reply), args.mount, out=f)
    finally:
        if f is not None:
            f.close()
    print(json.dumps(summary))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
