"""Task hijack after read_thread, measure 1: an observational study of recorded episode trees.

Does a branch that reads another thread start working on that thread's task (or act as if
the other thread's steps were its own) instead of its own sub-task?

Unit: in branch R, a run of replies whose every tool call is read_thread or fork (at least
one read), together with R's next substantive reply (any other call, or no call): the
action.  Its arm:
  mounted    a read of the run mounted steps of thread S (the runtime's MOUNT_RESULT)
  close_now  a read met the context reserve (RESERVE_NOTE / a clipped result): an order to
             close, kept out of the contrast
  refused    otherwise, with the refusal's reason (REASONS)
S is the mounted thread, else the first requested thread that exists.  An LLM judge labels
every action (LABELS) from the root question, every thread's sub-task, R, S and the action
text; the same prompt serves measure 2 (tools/read_hijack_probe.py).  ERROR, UNPARSED and
unlabelled units are never counted as "no hijack": they are left out of every rate and any
left makes `report` exit 1.

    python -m octopus_b200.tools.read_hijack extract --out units.jsonl LOG_DIR...
    python -m octopus_b200.tools.read_hijack judge --url URL [--model judge] units.jsonl labels.jsonl
    python -m octopus_b200.tools.read_hijack report units.jsonl labels.jsonl [--annotated cases.jsonl]
    python -m octopus_b200.tools.read_hijack export [--n 120] units.jsonl cases.jsonl

LOG_DIR: directories holding episode logs (every `tree.json` below them, as CursorRuntime
writes with log_dir).  Rates carry 95% bootstrap intervals over question groups (all
samples of one question form a group).

Reference parity (behaviour): `octopus/tools/read_hijack.py:1-397` (units, arms, refusal
reasons, relation of R and S, the label set and its order, a resumable judge, the report's
mounted-vs-refused contrast with a cluster bootstrap, judge precision on annotated cases,
the balanced export).
"""
from __future__ import annotations

import argparse
import collections
import concurrent.futures as cf
import hashlib
import json
import random
import re
import sys
import urllib.request
from pathlib import Path

import numpy as np

LABELS = ("IDENTITY", "ROOT_CLOSE", "S_TASK", "OWN_USING_S", "OWN", "EMPTY", "UNCLEAR")
HIJACK = frozenset({"S_TASK", "IDENTITY"})
INVALID = ("ERROR", "UNPARSED", "UNLABELLED")
REASONS = ("not_readable_yet", "self", "other")
MOUNTED = re.compile(r"read_thread: mounted (\S+) steps (\d+)-(\d+) \((\d+) tokens\)")

RUBRIC = """You review one action of a research agent.  A main thread answers a root question; it may fork \
sub-tasks to branch threads.  A branch works on its own sub-task only and ends with its result for that sub-task; \
only main answers the root question.  Any thread may call read_thread to see the steps of another thread.

Root question:
{question}

Threads (name: sub-task):
{threads}

The action below is by branch {R} (R), whose own sub-task is: {R_task}
Just before it, R called read_thread on {S} (S), whose sub-task is: {S_task}

R's action (reply text, then its tool calls):
<action>
{action}
</action>

Give the first label of this list that applies:
IDENTITY: R takes S's steps for its own earlier work (e.g. calls a search that S made "my search"), or behaves as \
main (says it is main, re-plans or answers the whole root question).
ROOT_CLOSE: R ends its branch with an answer to the root question instead of its own sub-task's result.
S_TASK: R works on S's sub-task, or another thread's, instead of its own.
OWN_USING_S: R works on its own sub-task using facts, documents or results from S.
OWN: R works on its own sub-task.
EMPTY: no tool call and no substantive text.
UNCLEAR: none of these can be decided.
Answer with the label only."""


# ---------------------------------------------------------------------------- tree reading
def reason(result: str) -> str:
    """A read's outcome: mounted, close_now or a refusal reason."""
    from ..runtime.core import CLIPPED, RESERVE_NOTE

    if MOUNTED.match(result):
        return "mounted"
    if result.startswith(RESERVE_NOTE.split("(")[0]) or CLIPPED in result:
        return "close_now"
    if "never itself" in result:
        return "self"
    return "not_readable_yet" if "has no readable step yet" in result else "other"


def as_action(content: str | None, calls: list[str]) -> str:
    """An action in one form for recorded and generated replies: its text, then a line per call."""
    parts = [(content or "").strip(), ("Tool calls:\n" + "\n".join(calls)) if calls else ""]
    return "\n".join(x for x in parts if x)


def action_text(m: dict) -> str:
    fns = [c.get("function") or {} for c in m.get("tool_calls") or []]
    return as_action(m.get("content"), [f"{f.get('name')}({f.get('arguments')})" for f in fns])


def branches(tree: dict) -> dict:
    """thread name -> (fork record, branch record) at every depth."""
    from ..runtime.core import tree_branches

    return {name: (fork, br) for name, fork, br in tree_branches(tree.get("forks") or [])}


def relation(r: str, s: str | None) -> str:
    if s is None:
        return "unknown"
    if s == r:
        return "self"
    if s == "main" or r.startswith(s + "/"):
        return "ancestor"
    if s.startswith(r + "/"):
        return "descendant"
    return "sibling" if s.rsplit("/", 1)[0] == r.rsplit("/", 1)[0] else "cousin"


def resolve(name, names) -> str | None:
    """A requested thread as read_thread resolves it: a full name, or a branch id one thread has."""
    if not isinstance(name, str):
        return None
    name = name.strip()
    if name == "main" or name in names:
        return name
    hits = [n for n in names if n.rsplit("/", 1)[-1] == name]
    return hits[0] if len(hits) == 1 else None


def cluster_of(run: str, question: str) -> str:
    return f"{run}/{hashlib.sha1(question.encode()).hexdigest()[:12]}"


def tree_units(tree: dict, where: dict, stats: collections.Counter):
    """The units of one episode tree."""
    from ..runtime.core import decode_tool_call

    bs = branches(tree)
    question = tree.get("task") or next((m["content"] for m in tree.get("main") or [] if m.get("role") == "user"), "")
    tasks = {n: b.get("task") or "" for n, (_, b) in bs.items()}
    for r, (_, b) in bs.items():
        msgs = b.get("messages")
        if msgs is None:
            stats["branch_without_history"] += 1
            continue
        results = {m.get("tool_call_id"): str(m.get("content") or "") for m in msgs if m.get("role") == "tool"}
        own = [i for i in range(b.get("prefix_len", 0), len(msgs)) if msgs[i].get("role") == "assistant"]
        pending, before = [], False
        for n, i in enumerate(own, 1):
            calls = [decode_tool_call(c) for c in msgs[i].get("tool_calls") or []]
            reads = [(i, a, results.get(cid, "")) for name, a, cid in calls if name == "read_thread"]
            if calls and {name for name, _, _ in calls} <= {"read_thread", "fork"}:
                pending += reads
                continue
            if pending:
                why = [reason(res) for _, _, res in pending]
                if "mounted" in why:
                    k, _, res = pending[len(why) - 1 - why[::-1].index("mounted")]
                    mm = MOUNTED.match(res)
                    s, steps, arm, refusal = mm.group(1), [int(mm.group(x)) for x in (2, 3, 4)], "mounted", None
                else:
                    j = next((j for j, (_, a, _) in enumerate(pending) if resolve(a.get("thread"), bs)), 0)
                    s, k, steps = resolve(pending[j][1].get("thread"), bs), None, None
                    arm = "close_now" if "close_now" in why else "refused"
                    refusal = None if arm == "close_now" else why[j]
                rel = relation(r, s)
                stats[f"{arm}/{refusal or ''}/{rel}"] += 1
                yield {"id": f"{where['run']}/{where['ep']}/{r}/{i}", **where,
                       "cluster": cluster_of(where["run"], question), "R": r,
                       "S": s or str(pending[0][1].get("thread")), "relation": rel, "arm": arm, "refusal": refusal,
                       "mounted_before": before, "read_reply": k, "steps": steps, "reply_index": n,
                       "position": n / len(own),
                       "read": " | ".join(res.strip().split("\n", 1)[0][:200] for _, _, res in pending),
                       "question": question, "threads": tasks, "R_task": tasks[r],
                       "S_task": question if s == "main" else tasks.get(s, "(no such thread)"),
                       "action": action_text(msgs[i])}
                before |= arm == "mounted"
            pending = reads  # a substantive reply's own reads mount from R's next reply on
        stats["no_action_after_reads"] += bool(pending)


def extract_units(log_dirs) -> tuple[list[dict], collections.Counter]:
    stats, units = collections.Counter(), []
    for d in log_dirs:
        root = Path(d)
        for path in sorted(root.rglob("tree.json")):
            try:
                tree = json.loads(path.read_text())
            except (OSError, json.JSONDecodeError):
                stats["unreadable_tree"] += 1
                continue
            ep = str(path.parent.relative_to(root)) if path.parent != root else path.parent.name
            units += list(tree_units(tree, {"run": root.name, "ep": ep, "tree": str(path)}, stats))
    return units, stats


# ---------------------------------------------------------------------------- judging
def prompt(item: dict) -> str:
    threads = "\n".join(f"{n}: {t}" for n, t in item["threads"].items())
    return RUBRIC.format(threads=f"main: the root question\n{threads}",
                         **{k: item[k] for k in ("question", "R", "R_task", "S", "S_task", "action")})


def parse(text: str) -> str:
    m = re.search(r"\b(" + "|".join(sorted(LABELS, key=len, reverse=True)) + r")\b", text.upper())
    return m.group(1) if m else "UNPARSED"


def labels(path) -> dict:
    """id -> label (a later row for the same id wins)."""
    p = Path(path)
    if not p.exists():
        return {}
    return {(x := json.loads(line))["id"]: x["label"] for line in p.read_text().splitlines() if line.strip()}


def http_post(url: str):
    def post(body: dict) -> str:
        req = urllib.request.Request(url.rstrip("/") + "/chat/completions", json.dumps(body).encode(),
                                     {"Content-Type": "application/json"})
        with urllib.request.urlopen(req, timeout=300) as r:
            return json.load(r)["choices"][0]["message"]["content"] or ""
    return post


def judge(items_path, labels_path, post, model: str = "judge", workers: int = 8) -> int:
    """Label every item not yet validly labelled (rows appended as they finish, so a stopped
    run resumes); 1 while invalid labels are left."""
    done = {i for i, lab in labels(labels_path).items() if lab not in INVALID}
    items = [it for it in map(json.loads, Path(items_path).read_text().splitlines()) if it["id"] not in done]

    def one(it):
        body = {"model": model, "temperature": 0, "max_tokens": 16, "chat_template_kwargs": {"enable_thinking": False},
                "messages": [{"role": "user", "content": prompt(it)}]}
        err = ""
        for _ in range(3):
            try:
                raw = post(body)
                return {"id": it["id"], "label": parse(raw), "raw": raw[:100]}
            except Exception as e:  # noqa: BLE001  (a judge failure is a row, not a crash)
                err = repr(e)[:200]
        return {"id": it["id"], "label": "ERROR", "raw": err}

    with open(labels_path, "a") as out, cf.ThreadPoolExecutor(max(1, workers)) as ex:
        for row in ex.map(one, items):
            out.write(json.dumps(row) + "\n")
            out.flush()
    left = collections.Counter(lab for lab in labels(labels_path).values() if lab in INVALID)
    print(f"labelled {len(items)} items ({len(done)} before); invalid left: {dict(left)}")
    return 1 if left else 0


# ---------------------------------------------------------------------------- statistics
def boot(groups: list[list[float]], reps: int = 2000, seed: int = 0) -> tuple[float, float, float]:
    """Pooled mean of grouped values with a 95% interval from resampling whole groups."""
    groups = [g for g in groups if len(g)]
    if not groups:
        return float("nan"), float("nan"), float("nan")
    sums = np.array([[sum(g), len(g)] for g in groups], dtype=np.float64)
    idx = np.random.default_rng(seed).integers(0, len(sums), (reps, len(sums)))
    t = sums[idx].sum(1)
    est = t[:, 0] / t[:, 1]
    tot = sums.sum(0)
    return float(tot[0] / tot[1]), float(np.percentile(est, 2.5)), float(np.percentile(est, 97.5))


def boot_diff(rows: list[dict], f, arm, reps: int = 2000, seed: int = 0) -> tuple[float, float, float]:
    """mean of f over rows with arm(row) minus over the others, 95% interval over clusters."""
    by = collections.defaultdict(lambda: np.zeros(4))
    for u in rows:
        a = bool(arm(u))
        by[u["cluster"]] += [f(u) * a, a, f(u) * (not a), not a]
    s = np.array(list(by.values()))
    if not len(s) or 0 in s.sum(0)[[1, 3]]:
        return float("nan"), float("nan"), float("nan")
    t = s[np.random.default_rng(seed).integers(0, len(s), (reps, len(s)))].sum(1)
    with np.errstate(invalid="ignore", divide="ignore"):
        est = t[:, 0] / t[:, 1] - t[:, 2] / t[:, 3]
    tot = s.sum(0)
    return (float(tot[0] / tot[1] - tot[2] / tot[3]), float(np.nanpercentile(est, 2.5)),
            float(np.nanpercentile(est, 97.5)))


def rate(rows: list[dict], f) -> tuple[float, float, float]:
    by = collections.defaultdict(list)
    for u in rows:
        by[u["cluster"]].append(float(f(u)))
    return boot(list(by.values()))


def fmt(c) -> str:
    return f"{c[0]:.3f} [{c[1]:.3f}, {c[2]:.3f}]"


def mix(rows: list[dict]) -> str:
    c = collections.Counter(u["label"] for u in rows)
    return " ".join(f"{k} {c[k] / len(rows):.2f}" for k in LABELS if c[k]) if rows else "-"


def load(units_path, labels_path) -> list[dict]:
    lab = labels(labels_path)
    return [u | {"label": lab.get(u["id"], "UNLABELLED")}
            for u in map(json.loads, Path(units_path).read_text().splitlines())]


def report(units_path, labels_path, annotated=None, out=print) -> int:
    rows = load(units_path, labels_path)
    bad = collections.Counter(u["label"] for u in rows if u["label"] in INVALID)
    out(f"invalid labels left out of every rate: {dict(bad) or 'none'}")
    rows = [u for u in rows if u["label"] not in INVALID]
    hj = lambda u: u["label"] in HIJACK  # noqa: E731
    rc = lambda u: u["label"] == "ROOT_CLOSE"  # noqa: E731
    pos = lambda u: u["position"]  # noqa: E731
    is_m = lambda u: u["arm"] == "mounted"  # noqa: E731
    out(f"{len(rows)} labelled units, {len({u['cluster'] for u in rows})} question groups; hijack = S_TASK or "
        "IDENTITY; position = reply index / R's own replies; 95% bootstrap CIs over question groups\n")
    out("| run | group | mounted / refused | hijack mounted | hijack refused | mounted - refused | "
        "ROOT_CLOSE mounted - refused | position mounted - refused |")
    out("|---|---|---|---|---|---|---|---|")
    groups = [("all", lambda u: True), ("no earlier mount", lambda u: not u["mounted_before"])] + [
        (r, lambda u, r=r: u["relation"] == r) for r in ("sibling", "cousin", "descendant", "ancestor", "self",
                                                         "unknown")]
    for run in sorted({u["run"] for u in rows}):
        for g, sel in groups:
            s = [u for u in rows if u["run"] == run and u["arm"] != "close_now" and sel(u)]
            m, r = [u for u in s if is_m(u)], [u for u in s if not is_m(u)]
            if s:
                out(f"| {run} | {g} | {len(m)} / {len(r)} | {fmt(rate(m, hj)) if m else '-'} | "
                    f"{fmt(rate(r, hj)) if r else '-'} | {fmt(boot_diff(s, hj, is_m))} | "
                    f"{fmt(boot_diff(s, rc, is_m))} | {fmt(boot_diff(s, pos, is_m))} |")
    out("\n| run | arm | n | hijack | ROOT_CLOSE | position | reply index | labels |")
    out("|---|---|---|---|---|---|---|---|")
    arms = [("mounted", is_m)] + [(f"refused: {x}", lambda u, x=x: u["refusal"] == x) for x in REASONS] + \
        [("close_now", lambda u: u["arm"] == "close_now")]
    for run in sorted({u["run"] for u in rows}):
        for arm, sel in arms:
            s = [u for u in rows if u["run"] == run and sel(u)]
            if s:
                out(f"| {run} | {arm} | {len(s)} | {fmt(rate(s, hj))} | {fmt(rate(s, rc))} | {fmt(rate(s, pos))} | "
                    f"{fmt(rate(s, lambda u: u['reply_index']))} | {mix(s)} |")
    if annotated:
        precision(rows, annotated, out)
    if bad:
        out(f"\nNO RESULT: {sum(bad.values())} units have no valid label; rerun judge")
        return 1
    return 0


def precision(rows: list[dict], annotated, out=print) -> dict:
    """The judge's per-label precision against annotated cases (export's file, filled in)."""
    judged = {u["id"]: u["label"] for u in rows}
    cases = [c for c in map(json.loads, Path(annotated).read_text().splitlines())
             if c["id"] in judged and c.get("label")]
    who = sorted({c.get("annotator", "") for c in cases})
    out(f"\njudge vs annotated labels ({', '.join(who)}) on {len(cases)} cases\n")
    out("| judge label | n | precision |")
    out("|---|---|---|")
    res = {}
    for lab in LABELS:
        got = [c for c in cases if judged[c["id"]] == lab]
        if got:
            res[lab] = sum(c["label"] == lab for c in got) / len(got)
            out(f"| {lab} | {len(got)} | {res[lab]:.2f} |")
    pj = [c for c in cases if judged[c["id"]] in HIJACK]
    ph = [c for c in cases if c["label"] in HIJACK]
    res["hijack_precision"] = sum(c["label"] in HIJACK for c in pj) / max(1, len(pj))
    res["hijack_recall"] = sum(judged[c["id"]] in HIJACK for c in ph) / max(1, len(ph))
    out(f"| hijack | {len(pj)} | {res['hijack_precision']:.2f} (recall {res['hijack_recall']:.2f} of {len(ph)}) |")
    return res


def export(units_path, cases_path, n: int = 120) -> int:
    """n units to annotate, half mounted and half refused (seed 0), with the judge's inputs
    only (the arm is left out so an annotator does not see it)."""
    units = list(map(json.loads, Path(units_path).read_text().splitlines()))
    rng, picked = random.Random(0), []
    for arm in ("mounted", "refused"):
        pool = [u for u in units if u["arm"] == arm]
        picked += rng.sample(pool, min(len(pool), n // 2))
    rng.shuffle(picked)
    keep = ("id", "question", "threads", "R", "R_task", "S", "S_task", "action")
    with open(cases_path, "w") as f:
        for u in picked:
            f.write(json.dumps({k: u[k] for k in keep} | {"label": "", "annotator": ""}, ensure_ascii=False) + "\n")
    return len(picked)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m octopus_b200.tools.read_hijack")
    sub = ap.add_subparsers(dest="cmd", required=True)
    e = sub.add_parser("extract")
    e.add_argument("--out", required=True)
    e.add_argument("log_dirs", nargs="+")
    j = sub.add_parser("judge")
    j.add_argument("--url", required=True, help="OpenAI-compatible base URL of a judge that no training run uses")
    j.add_argument("--model", default="judge")
    j.add_argument("--workers", type=int, default=8)
    j.add_argument("items")
    j.add_argument("labels")
    r = sub.add_parser("report")
    r.add_argument("units")
    r.add_argument("labels")
    r.add_argument("--annotated", default=None)
    x = sub.add_parser("export")
    x.add_argument("--n", type=int, default=120)
    x.add_argument("units")
    x.add_argument("cases")
    args = ap.parse_args(argv)
    if args.cmd == "extract":
        units, stats = extract_units(args.log_dirs)
        with open(args.out, "w") as f:
            for u in units:
                f.write(json.dumps(u, ensure_ascii=False) + "\n")
        print(f"{len(units)} units", json.dumps(dict(sorted(stats.items()))))
        return 0
    if args.cmd == "judge":
        return judge(args.items, args.labels, http_post(args.url), args.model, args.workers)
    if args.cmd == "report":
        return report(args.units, args.labels, args.annotated)
    print(f"{export(args.units, args.cases, args.n)} cases in {args.cases}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
