"""Task hijack after read_thread, measure 2: a counterfactual probe at recorded mount points.

At each mounted unit of measure 1 (tools/read_hijack.py), R's history through the reply
whose read mounted, plus that reply's tool results, is rebuilt as tokens and R's next reply
is sampled again on the engine under three conditions:
  none   R's history as recorded, nothing mounted (the read's result line stays)
  text   the same, with S's mounted steps appended as text to the read's result
  mount  `none` plus the mount of S's steps, as the runtime reads (rule K2): S's rows as S
         computed them, inside R's attention
All three continue one prefill-only cursor of R's history; the mount names a prefill-only
cursor of S's history over the token range of the read's steps (from step lo's reply to the
end of step hi's reply).  Under K2 R's tokens continue at max(len(R), range end), so each
point records jump = max(0, end - len(R)) and the report stratifies by it.  Rendering is
the chat template (positions may differ from the run's by a per-thread constant, the same
for every condition); range_minus_read records the rendered range minus the read's token
count.  Skipped (counted): a point whose R mounted before, whose S mounted anything before
the range end, or whose S rewound.  Each sample becomes a judge item in measure 1's form
(`python -m octopus_b200.tools.read_hijack judge`).

    python -m octopus_b200.tools.read_hijack_probe run --checkpoint NAME=HF_DIR[,NAME=HF_DIR]
        [--preset qwen2.5-7b] [--n 300] [--samples 4] units.jsonl items.jsonl
    python -m octopus_b200.tools.read_hijack_probe report items.jsonl labels.jsonl

`run` appends to items.jsonl and skips (point, checkpoint) pairs already there.  The first
checkpoint is the report's reference and gives the tokenizer; with several, the report gives each one's
(mount - none) minus the reference's.

Reference parity (behaviour): `octopus/tools/read_hijack_probe.py:1-282` (the three
conditions, the K2 jump, skip rules, judge items, the per-point means, the cluster bootstrap
and the pre-registered decision rule: mount hijacks when the lower bound of mount - none is
above 0.05, no hijack when its upper bound is at most 0.05).
"""
from __future__ import annotations

import argparse
import collections
import json
import random
import re
import sys
from pathlib import Path

from .read_hijack import HIJACK, INVALID, LABELS, MOUNTED, action_text, as_action, boot, branches, fmt, labels

CONDITIONS = ("none", "text", "mount")
TEXT = "\n\nThe full text of these steps:\n"


class Skip(Exception):
    pass


def text_of(msgs: list[dict]) -> str:
    return "\n".join(f"[{m['role']}] " + (action_text(m) if m["role"] == "assistant" else str(m.get("content") or ""))
                     for m in msgs)


def _mounted_in(msgs: list[dict]) -> bool:
    return any(m.get("role") == "tool" and MOUNTED.match(str(m.get("content") or "")) for m in msgs)


def point(u: dict, tok) -> dict:
    """Token sequences of one mount point; Skip when it cannot be rebuilt."""
    tree = json.loads(Path(u["tree"]).read_text())
    bs = branches(tree)
    r_rec = bs[u["R"]][1]
    rmsgs, rtools, k = r_rec["messages"], r_rec.get("tools"), u["read_reply"]
    t = next((j for j in range(k + 1, len(rmsgs)) if rmsgs[j]["role"] != "tool"), len(rmsgs))
    hist = rmsgs[:t]
    if _mounted_in(rmsgs[:k]):
        raise Skip("reader mounted before")
    if u["S"] == "main":
        smsgs, s_prefix, stools = tree.get("main") or [], 0, tree.get("tools")
    else:
        s_rec = bs[u["S"]][1]
        if s_rec.get("rewinds"):
            raise Skip("source rewound")
        smsgs, s_prefix, stools = s_rec["messages"], s_rec.get("prefix_len", 0), s_rec.get("tools")
    lo, hi, n = u["steps"]
    own = [i for i in range(s_prefix, len(smsgs)) if smsgs[i]["role"] == "assistant"]
    if not smsgs or hi >= len(own):
        raise Skip("steps not in the source's history")
    i_lo, i_hi = own[lo], own[hi]
    a_msgs = smsgs[:i_hi + 1]
    if _mounted_in(a_msgs):
        raise Skip("source mounted before the range end")

    def ids(msgs, tools, gen=False):
        return tok.encode(tok.render(msgs, tools, gen))

    a, pre = ids(a_msgs, stools), ids(smsgs[:i_lo], stools, True)
    if a[:len(pre)] != pre:
        raise Skip("source rendering is not a prefix")
    s, e = len(pre), len(a)
    j = next(j for j in range(k + 1, t) if MOUNTED.match(str(hist[j].get("content") or "")))
    with_text = hist[:j] + [{**hist[j], "content": hist[j]["content"] + TEXT + text_of(smsgs[i_lo:i_hi + 1])}] + \
        hist[j + 1:]
    b, full, full_text = ids(rmsgs[:k + 1], rtools), ids(hist, rtools, True), ids(with_text, rtools, True)
    if full[:len(b)] != b or full_text[:len(b)] != b:
        raise Skip("reader rendering is not a prefix")
    return {"a": a, "s": s, "e": e, "b": b, "delta": {"none": full[len(b):], "text": full_text[len(b):]},
            "jump": max(0, e - len(b)), "range_minus_read": e - s - n}


def select_points(units: list[dict], tok, n: int, per_episode: int = 2):
    """Mounted units in shuffled order (seed 0) until n points, at most `per_episode` each."""
    units = [u for u in units if u["arm"] == "mounted"]
    random.Random(0).shuffle(units)
    points, skipped, per_ep = [], collections.Counter(), collections.Counter()
    for u in units:
        if len(points) == n:
            break
        if per_ep[u["ep"]] >= per_episode:
            continue
        try:
            points.append((u, point(u, tok)))
            per_ep[u["ep"]] += 1
        except Skip as x:
            skipped[str(x)] += 1
    return points, skipped


def parse_reply(tok, output_ids: list[int]) -> tuple[str, set]:
    """A sampled reply in measure 1's action form, and the names of its tool calls."""
    from ..serving.chat import parse_tool_calls

    text = re.sub(r"<think>.*?</think>", "", tok.decode([i for i in output_ids if i not in tok.stop_ids]), flags=re.S)
    content, calls = parse_tool_calls(text)
    fns = [c["function"] for c in calls]
    return as_action(content, [f"{f['name']}({f['arguments']})" for f in fns]), {f["name"] for f in fns}


def sample_point(engine, tok, u: dict, p: dict, ckpt: str, samples: int, temperature: float,
                 max_tokens: int) -> list[dict]:
    """Judge items of one (point, checkpoint): `samples` replies per condition."""
    from ..serving.engine import GenInput

    tag = f"rhp/{ckpt}/{u['id']}"
    ca, cb = f"{tag}/a", f"{tag}/b"
    engine.generate([GenInput(p["a"], max_new_tokens=0, prefill_only=True, cursor_id=ca),
                     GenInput(p["b"], max_new_tokens=0, prefill_only=True, cursor_id=cb)])
    rows = []
    try:
        for cond in CONDITIONS:
            mount = [(ca, p["s"], p["e"])] if cond == "mount" else []
            gens = [GenInput(p["delta"]["text" if cond == "text" else "none"], cursor=cb, mount=mount,
                             mount_rule="K2", max_new_tokens=max_tokens, temperature=temperature,
                             stop_ids=tuple(tok.stop_ids), keep_cursor=False) for _ in range(samples)]
            for i, o in enumerate(engine.generate(gens)):
                action, names = parse_reply(tok, o.output_ids)
                rows.append({k: u[k] for k in ("question", "threads", "R", "R_task", "S", "S_task", "relation", "run",
                                                "cluster")}
                            | {"id": f"{u['id']}|{ckpt}|{cond}|{i}", "point": u["id"], "ckpt": ckpt, "cond": cond,
                               "sample": i, "action": action, "jump": p["jump"],
                               "range_minus_read": p["range_minus_read"],
                               "skip": bool(names) and names <= {"read_thread", "fork"}})
    finally:
        engine.release_cursor(ca)
        engine.release_cursor(cb)
    return rows


def run(engine, tok, units: list[dict], items_path, ckpt: str, n: int = 300, samples: int = 4,
        temperature: float = 0.7, max_tokens: int = 4096) -> dict:
    points, skipped = select_points(units, tok, n)
    p_items = Path(items_path)
    done = {(x["point"], x["ckpt"]) for x in map(json.loads, p_items.read_text().splitlines())} \
        if p_items.exists() else set()
    written = failed = 0
    with open(items_path, "a") as out:
        for u, p in points:
            if (u["id"], ckpt) in done:
                continue
            try:
                rows = sample_point(engine, tok, u, p, ckpt, samples, temperature, max_tokens)
            except Exception as e:  # noqa: BLE001  (a failed pair is retried by the next run)
                print(f"failed {u['id']} {ckpt}: {e!r}"[:400], flush=True)
                failed += 1
                continue
            out.writelines(json.dumps(r, ensure_ascii=False) + "\n" for r in rows)
            out.flush()
            written += 1
    return {"points": len(points), "skipped": dict(skipped), "written": written, "failed": failed,
            "before": len(done)}


def report(items_path, labels_path, out=print) -> int:
    lab = labels(labels_path)
    items = [it | {"label": lab.get(it["id"], "UNLABELLED")}
             for it in map(json.loads, Path(items_path).read_text().splitlines())]
    bad = collections.Counter(it["label"] for it in items if it["label"] in INVALID)
    out(f"invalid labels left out of every rate: {dict(bad) or 'none'}")
    # per (checkpoint, point, condition): the mean over its valid samples; a reply that only
    # reads or forks is never a hijack
    score = {"hijack": lambda it: it["label"] in HIJACK and not it["skip"],
             "root_close": lambda it: it["label"] == "ROOT_CLOSE" and not it["skip"],
             "read_or_fork_only": lambda it: it["skip"]}
    by = collections.defaultdict(list)
    for it in items:
        if it["label"] not in INVALID:
            by[it["ckpt"], it["point"], it["cond"]].append(it)
    ckpts = list(dict.fromkeys(it["ckpt"] for it in items))
    pts = {it["point"]: it for it in items}
    strata = {"all": lambda p: True, "sibling": lambda p: p["relation"] == "sibling",
              "cousin": lambda p: p["relation"] == "cousin", "descendant": lambda p: p["relation"] == "descendant",
              "K2 jump": lambda p: p["jump"] > 0, "no jump": lambda p: p["jump"] == 0}

    def values(ck, f, cond, ref=None, ck0=None, sel=strata["all"]):
        """per cluster, per point: f's mean under cond (minus under ref; minus the same at ck0)"""
        res = collections.defaultdict(list)
        for p, it in pts.items():
            if not sel(it) or not all((k, p, c) in by for k in {ck, ck0} - {None} for c in CONDITIONS):
                continue
            m = lambda c, k: sum(map(f, by[k, p, c])) / len(by[k, p, c])  # noqa: E731
            v = m(cond, ck) - (m(ref, ck) if ref else 0)
            if ck0:
                v -= m(cond, ck0) - (m(ref, ck0) if ref else 0)
            res[it["cluster"]].append(v)
        return list(res.values())

    out(f"{len(pts)} mount points ({sum(p['jump'] > 0 for p in pts.values())} with a K2 jump), "
        f"{len({p['cluster'] for p in pts.values()})} question groups, checkpoints {ckpts}\n")
    out("| checkpoint | stratum | score | none | text | mount | mount - none | text - none | mount - text |")
    out("|---|---|---|---|---|---|---|---|---|")
    for ck in ckpts:
        for st, sel in strata.items():
            for name, f in score.items():
                if not values(ck, f, "none", sel=sel):
                    continue
                cells = [fmt(boot(values(ck, f, c, sel=sel))) for c in CONDITIONS]
                diffs = [fmt(boot(values(ck, f, a, b, sel=sel)))
                         for a, b in (("mount", "none"), ("text", "none"), ("mount", "text"))]
                out(f"| {ck} | {st} | {name} | " + " | ".join(cells + diffs) + " |")
    out("\nlabel mix:")
    for ck in ckpts:
        for cond in CONDITIONS:
            c = collections.Counter(it["label"] for it in items
                                    if it["ckpt"] == ck and it["cond"] == cond and it["label"] not in INVALID)
            tot = max(1, sum(c.values()))
            out(f"  {ck} {cond}: " + " ".join(f"{k} {c[k] / tot:.2f}" for k in LABELS if c[k]))
    if bad:
        out(f"\nNO DECISION: {sum(bad.values())} samples have no valid label; rerun judge")
        return 1
    out("\ndecision (hijack):")
    hj = score["hijack"]
    for ck in ckpts:
        d = boot(values(ck, hj, "mount", "none"))
        verdict = "the mount hijacks" if d[1] > 0.05 else "no mount hijack" if d[2] <= 0.05 else "inconclusive"
        out(f"  {ck}: mount - none {fmt(d)} -> {verdict}; text - none {fmt(boot(values(ck, hj, 'text', 'none')))}")
        if ck != ckpts[0]:
            t = boot(values(ck, hj, "mount", "none", ck0=ckpts[0]))
            out(f"    (mount - none) at {ck} minus at {ckpts[0]}: {fmt(t)} -> "
                + ("training raised the mount's hijack" if t[1] > 0 else "training lowered it" if t[2] < 0
                   else "no change shown"))
    return 0


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m octopus_b200.tools.read_hijack_probe")
    sub = ap.add_subparsers(dest="cmd", required=True)
    r = sub.add_parser("run")
    r.add_argument("--checkpoint", required=True, help="NAME=HF_DIR[,NAME=HF_DIR...]; the first is the reference")
    r.add_argument("--preset", default="qwen2.5-7b")
    r.add_argument("--n", type=int, default=300)
    r.add_argument("--samples", type=int, default=4)
    r.add_argument("--temperature", type=float, default=0.7)
    r.add_argument("--max-tokens", type=int, default=4096)
    r.add_argument("--kv-gb", type=float, default=16.0)
    r.add_argument("units")
    r.add_argument("items")
    p = sub.add_parser("report")
    p.add_argument("items")
    p.add_argument("labels")
    args = ap.parse_args(argv)
    if args.cmd == "report":
        return report(args.items, args.labels)

    from ..eval.search_eval import build_service
    from ..models.decoder import load_hf

    ckpts = [c.split("=", 1) for c in args.checkpoint.split(",")]
    units = list(map(json.loads, Path(args.units).read_text().splitlines()))
    svc, eng = build_service(args.preset, ckpts[0][1], args.kv_gb)
    failed = 0
    for i, (name, path) in enumerate(ckpts):
        if i:
            load_hf(eng.w, path)
            eng.bump_version()
            eng.reset()
        res = run(eng, svc.tok, units, args.items, name, args.n, args.samples, args.temperature, args.max_tokens)
        print(json.dumps({"checkpoint": name, **res}), flush=True)
        failed += res["failed"]
    return 1 if failed else 0


if __name__ == "__main__":
    sys.exit(main())
