"""Task hijack after read_thread, measure 2: a counterfactual probe at logged mount points.

For each mounted unit of measure 1 (tools/read_hijack.py), R's history up to and including
the reply whose read mounted S (with that reply's tool results) is rebuilt as tokens, and
R's next reply is sampled again on the engine under three conditions:
  none   R's history as logged, with nothing mounted (the read's result line stays)
  text   the same history with S's mounted steps appended as text to the read's result
  mount  `none` plus the mount of S's steps as the runtime does it (rule K2): S's rows,
         computed by S, inside R's attention
All three continue one prefill-only cursor of R's history.  The mount names a prefill-only
cursor of S's history over the token range of the read's steps (from step lo's reply to the
end of step hi's reply).  Under K2 R's tokens continue at max(len(R), range end), so each
point records jump = max(0, end - len(R)) and the report stratifies by it.  Rendering uses
the chat template (positions may differ from the run's by a per-thread constant, the same
in every condition); range_minus_read is the rendered range minus the read's logged token
count.  A point is skipped (and counted) when R mounted earlier, when S mounted anything
before the range end, or when S rewound.  Every sample becomes a judge item in measure 1's
form (`python -m octopus_b200.tools.read_hijack judge`).

    python -m octopus_b200.tools.read_hijack_probe run --checkpoint NAME=HF_DIR[,NAME=HF_DIR]
        [--preset qwen2.5-7b] [--n 300] [--samples 4] units.jsonl items.jsonl
    python -m octopus_b200.tools.read_hijack_probe report items.jsonl labels.jsonl

`run` appends to items.jsonl and skips (point, checkpoint) pairs it already holds.  The
first checkpoint is the reference (and gives the tokenizer); with several, the report
gives each one's (mount - none) minus the reference's.

Reference parity (behaviour): `octopus/tools/read_hijack_probe.py:1-282` (the three
conditions, the K2 jump, the skip rules, judge items, per-point means, cluster bootstrap,
and the pre-registered decision: the mount hijacks when the lower bound of mount - none is
above 0.05, it does not when the upper bound is at most 0.05).
"""
from __future__ import annotations

import argparse
import collections
import json
import random
import re
import sys
from pathlib import Path

from .cluster_boot import ci_text, pooled_ci
from .read_hijack import HIJACK, INVALID, LABELS, MOUNTED, action_text, as_action, branches, labels

CONDITIONS = ("none", "text", "mount")
TEXT = "\n\nThe full text of these steps:\n"
DECISION_MARGIN = 0.05


class SkipPoint(Exception):
    """A mount point that cannot be rebuilt faithfully (the reason is the message)."""


def transcript(msgs: list[dict]) -> str:
    """Messages as plain text (the `text` condition's copy of S's steps)."""
    lines = []
    for m in msgs:
        body = action_text(m) if m["role"] == "assistant" else str(m.get("content") or "")
        lines.append(f"[{m['role']}] {body}")
    return "\n".join(lines)


def _has_mount(msgs: list[dict]) -> bool:
    return any(m.get("role") == "tool" and MOUNTED.match(str(m.get("content") or "")) for m in msgs)


class _PointBuilder:
    """Token sequences of one mount point, from the unit and its logged tree."""

    def __init__(self, unit: dict, tok):
        self.u, self.tok = unit, tok
        self.tree = json.loads(Path(unit["tree"]).read_text())
        self.threads = branches(self.tree)

    def ids(self, msgs, tools, add_generation_prompt=False) -> list[int]:
        return self.tok.encode(self.tok.render(msgs, tools, add_generation_prompt))

    def source(self):
        """(S's messages, index of its first own message, S's tools)."""
        if self.u["S"] == "main":
            return self.tree.get("main") or [], 0, self.tree.get("tools")
        rec = self.threads[self.u["S"]][1]
        if rec.get("rewinds"):
            raise SkipPoint("source rewound")
        return rec["messages"], rec.get("prefix_len", 0), rec.get("tools")

    def build(self) -> dict:
        reader = self.threads[self.u["R"]][1]
        rmsgs, rtools, k = reader["messages"], reader.get("tools"), self.u["read_reply"]
        if _has_mount(rmsgs[:k]):
            raise SkipPoint("reader mounted before")
        # R's history: through the reading reply and its tool results
        end = next((j for j in range(k + 1, len(rmsgs)) if rmsgs[j]["role"] != "tool"), len(rmsgs))
        history = rmsgs[:end]
        smsgs, s_first, stools = self.source()
        lo, hi, read_tokens = self.u["steps"]
        s_replies = [i for i in range(s_first, len(smsgs)) if smsgs[i]["role"] == "assistant"]
        if not smsgs or hi >= len(s_replies):
            raise SkipPoint("steps not in the source's history")
        first, last = s_replies[lo], s_replies[hi]
        if _has_mount(smsgs[:last + 1]):
            raise SkipPoint("source mounted before the range end")
        a = self.ids(smsgs[:last + 1], stools)
        head = self.ids(smsgs[:first], stools, True)
        if a[:len(head)] != head:
            raise SkipPoint("source rendering is not a prefix")
        s, e = len(head), len(a)
        at = next(j for j in range(k + 1, end) if MOUNTED.match(str(history[j].get("content") or "")))
        widened = dict(history[at])
        widened["content"] = history[at]["content"] + TEXT + transcript(smsgs[first:last + 1])
        with_text = history[:at] + [widened] + history[at + 1:]
        b = self.ids(rmsgs[:k + 1], rtools)
        plain, texted = self.ids(history, rtools, True), self.ids(with_text, rtools, True)
        if plain[:len(b)] != b or texted[:len(b)] != b:
            raise SkipPoint("reader rendering is not a prefix")
        return {"a": a, "s": s, "e": e, "b": b, "delta": {"none": plain[len(b):], "text": texted[len(b):]},
                "jump": max(0, e - len(b)), "range_minus_read": e - s - read_tokens}


def point(unit: dict, tok) -> dict:
    """Token sequences of one mount point (SkipPoint when it cannot be rebuilt)."""
    return _PointBuilder(unit, tok).build()


def select_points(units: list[dict], tok, n: int, per_episode: int = 2):
    """Mounted units in a seeded shuffle (seed 0), at most `per_episode` per episode,
    until n points are built; returns (points, skip reasons counted)."""
    pool = [u for u in units if u["arm"] == "mounted"]
    random.Random(0).shuffle(pool)
    points, skipped, taken = [], collections.Counter(), collections.Counter()
    for u in pool:
        if len(points) >= n:
            break
        if taken[u["ep"]] >= per_episode:
            continue
        try:
            p = point(u, tok)
        except SkipPoint as why:
            skipped[str(why)] += 1
            continue
        points.append((u, p))
        taken[u["ep"]] += 1
    return points, skipped


def parse_reply(tok, output_ids: list[int]) -> tuple[str, set]:
    """A sampled reply in measure 1's action form, and the names of its tool calls."""
    from ..serving.chat import parse_tool_calls

    text = tok.decode([i for i in output_ids if i not in tok.stop_ids])
    text = re.sub(r"<think>.*?</think>", "", text, flags=re.S)
    content, calls = parse_tool_calls(text)
    fns = [c["function"] for c in calls]
    return as_action(content, [f"{f['name']}({f['arguments']})" for f in fns]), {f["name"] for f in fns}


_CARRIED = ("question", "threads", "R", "R_task", "S", "S_task", "relation", "run", "cluster")


def sample_point(engine, tok, u: dict, p: dict, ckpt: str, samples: int, temperature: float,
                 max_tokens: int) -> list[dict]:
    """Judge items of one (point, checkpoint): `samples` replies under each condition."""
    from ..serving.engine import GenInput

    src_cursor, reader_cursor = f"rhp/{ckpt}/{u['id']}/a", f"rhp/{ckpt}/{u['id']}/b"
    engine.generate([GenInput(p["a"], max_new_tokens=0, prefill_only=True, cursor_id=src_cursor),
                     GenInput(p["b"], max_new_tokens=0, prefill_only=True, cursor_id=reader_cursor)])
    items = []
    try:
        for cond in CONDITIONS:
            delta = p["delta"]["text" if cond == "text" else "none"]
            mount = [(src_cursor, p["s"], p["e"])] if cond == "mount" else []
            reqs = [GenInput(delta, cursor=reader_cursor, mount=mount, mount_rule="K2", max_new_tokens=max_tokens,
                             temperature=temperature, stop_ids=tuple(tok.stop_ids), keep_cursor=False)
                    for _ in range(samples)]
            for i, res in enumerate(engine.generate(reqs)):
                action, names = parse_reply(tok, res.output_ids)
                item = {k: u[k] for k in _CARRIED}
                item.update(id=f"{u['id']}|{ckpt}|{cond}|{i}", point=u["id"], ckpt=ckpt, cond=cond, sample=i,
                            action=action, jump=p["jump"], range_minus_read=p["range_minus_read"],
                            skip=bool(names) and names <= {"read_thread", "fork"})
                items.append(item)
    finally:
        engine.release_cursor(src_cursor)
        engine.release_cursor(reader_cursor)
    return items


def run(engine, tok, units: list[dict], items_path, ckpt: str, n: int = 300, samples: int = 4,
        temperature: float = 0.7, max_tokens: int = 4096) -> dict:
    points, skipped = select_points(units, tok, n)
    path = Path(items_path)
    done = set()
    if path.exists():
        done = {(x["point"], x["ckpt"]) for x in map(json.loads, path.read_text().splitlines())}
    written = failed = 0
    with open(path, "a") as sink:
        for u, p in points:
            if (u["id"], ckpt) in done:
                continue
            try:
                rows = sample_point(engine, tok, u, p, ckpt, samples, temperature, max_tokens)
            except Exception as e:  # noqa: BLE001  (the pair stays missing; the next run retries it)
                print(f"failed {u['id']} {ckpt}: {e!r}"[:400], flush=True)
                failed += 1
                continue
            sink.writelines(json.dumps(r, ensure_ascii=False) + "\n" for r in rows)
            sink.flush()
            written += 1
    return {"points": len(points), "skipped": dict(skipped), "written": written, "failed": failed,
            "before": len(done)}


# ---------------------------------------------------------------------------- report
SCORES = {  # a reply that only reads or forks is never counted as a hijack
    "hijack": lambda it: it["label"] in HIJACK and not it["skip"],
    "root_close": lambda it: it["label"] == "ROOT_CLOSE" and not it["skip"],
    "read_or_fork_only": lambda it: it["skip"],
}
STRATA = {
    "all": lambda p: True,
    "sibling": lambda p: p["relation"] == "sibling",
    "cousin": lambda p: p["relation"] == "cousin",
    "descendant": lambda p: p["relation"] == "descendant",
    "K2 jump": lambda p: p["jump"] > 0,
    "no jump": lambda p: p["jump"] == 0,
}


class _Means:
    """Per (checkpoint, point, condition): the mean of a score over the valid samples;
    differences are taken per point, then grouped by question cluster."""

    def __init__(self, items: list[dict]):
        self.cells = collections.defaultdict(list)
        for it in items:
            if it["label"] not in INVALID:
                self.cells[it["ckpt"], it["point"], it["cond"]].append(it)
        self.points = {it["point"]: it for it in items}

    def _complete(self, ckpts, pid) -> bool:
        return all((ck, pid, c) in self.cells for ck in ckpts for c in CONDITIONS)

    def mean(self, score, ck, pid, cond) -> float:
        cell = self.cells[ck, pid, cond]
        return sum(map(score, cell)) / len(cell)

    def grouped(self, score, ck, cond, minus=None, base_ck=None, stratum=STRATA["all"]) -> list[list[float]]:
        ckpts = [ck] + ([base_ck] if base_ck else [])
        groups = collections.defaultdict(list)
        for pid, it in self.points.items():
            if not stratum(it) or not self._complete(ckpts, pid):
                continue

            def effect(k):
                v = self.mean(score, k, pid, cond)
                return v - self.mean(score, k, pid, minus) if minus else v
            v = effect(ck) - (effect(base_ck) if base_ck else 0.0)
            groups[it["cluster"]].append(v)
        return list(groups.values())


def _verdict(ci) -> str:
    if ci[1] > DECISION_MARGIN:
        return "the mount hijacks"
    if ci[2] <= DECISION_MARGIN:
        return "no mount hijack"
    return "inconclusive"


def report(items_path, labels_path, out=print) -> int:
    lab = labels(labels_path)
    items = [{**it, "label": lab.get(it["id"], "UNLABELLED")}
             for it in map(json.loads, Path(items_path).read_text().splitlines())]
    invalid = collections.Counter(it["label"] for it in items if it["label"] in INVALID)
    out(f"invalid labels left out of every rate: {dict(invalid) or 'none'}")
    means = _Means(items)
    ckpts = list(dict.fromkeys(it["ckpt"] for it in items))
    pts = means.points.values()
    out(f"{len(means.points)} mount points ({sum(p['jump'] > 0 for p in pts)} with a K2 jump), "
        f"{len({p['cluster'] for p in pts})} question groups, checkpoints {ckpts}\n")
    out("| checkpoint | stratum | score | none | text | mount | mount - none | text - none | mount - text |")
    out("|---|---|---|---|---|---|---|---|---|")
    pairs = (("mount", "none"), ("text", "none"), ("mount", "text"))
    for ck in ckpts:
        for sname, stratum in STRATA.items():
            for score_name, score in SCORES.items():
                if not means.grouped(score, ck, "none", stratum=stratum):
                    continue
                cells = [ci_text(pooled_ci(means.grouped(score, ck, c, stratum=stratum))) for c in CONDITIONS]
                cells += [ci_text(pooled_ci(means.grouped(score, ck, x, y, stratum=stratum))) for x, y in pairs]
                out(f"| {ck} | {sname} | {score_name} | " + " | ".join(cells) + " |")
    out("\nlabel mix:")
    for ck in ckpts:
        for cond in CONDITIONS:
            c = collections.Counter(it["label"] for it in items
                                    if it["ckpt"] == ck and it["cond"] == cond and it["label"] not in INVALID)
            total = max(1, sum(c.values()))
            out(f"  {ck} {cond}: " + " ".join(f"{k} {c[k] / total:.2f}" for k in LABELS if c[k]))
    if invalid:
        out(f"\nNO DECISION: {sum(invalid.values())} samples have no valid label; rerun judge")
        return 1
    out("\ndecision (hijack):")
    hijack = SCORES["hijack"]
    for ck in ckpts:
        d = pooled_ci(means.grouped(hijack, ck, "mount", "none"))
        t = pooled_ci(means.grouped(hijack, ck, "text", "none"))
        out(f"  {ck}: mount - none {ci_text(d)} -> {_verdict(d)}; text - none {ci_text(t)}")
        if ck != ckpts[0]:
            dd = pooled_ci(means.grouped(hijack, ck, "mount", "none", base_ck=ckpts[0]))
            change = ("training raised the mount's hijack" if dd[1] > 0 else
                      "training lowered it" if dd[2] < 0 else "no change shown")
            out(f"    (mount - none) at {ck} minus at {ckpts[0]}: {ci_text(dd)} -> {change}")
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
