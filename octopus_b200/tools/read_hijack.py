"""Task hijack after read_thread, measure 1: an observational study of logged episode trees.

Question: after a branch R reads another thread S, does R drift to S's task (or treat
S's steps as its own) instead of continuing its own sub-task?

Unit.  In branch R, a stretch of replies that only read or fork (at least one read)
followed by R's next substantive reply (any other call, or no call at all): that reply
is the unit's *action*.  Its arm:
  mounted    one of the stretch's reads mounted S's steps (the runtime's MOUNT_RESULT)
  close_now  a read hit the context reserve (the reserve refusal, or a clipped result):
             an order to close, kept out of the mounted-vs-refused contrast
  refused    otherwise; the refusal's reason is one of REASONS
S is the mounted thread (the last mount of the stretch), else the first requested thread
that exists.  A judge model labels every action with one of LABELS from the root question,
every thread's sub-task, R, S and the action text; measure 2 (tools/read_hijack_probe.py)
sends its samples through the same judge.  ERROR, UNPARSED and unlabelled units are never
read as "no hijack": they are left out of every rate, and while any is left `report`
exits 1.

    python -m octopus_b200.tools.read_hijack extract --out units.jsonl LOG_DIR...
    python -m octopus_b200.tools.read_hijack judge --url URL [--model judge] units.jsonl labels.jsonl
    python -m octopus_b200.tools.read_hijack report units.jsonl labels.jsonl [--annotated cases.jsonl]
    python -m octopus_b200.tools.read_hijack export [--n 120] units.jsonl cases.jsonl

LOG_DIR holds episode logs (every tree.json below it, as CursorRuntime writes them with
log_dir).  Intervals are 95% cluster-bootstrap intervals over question groups (all samples
of one question form a group).

Reference parity (behaviour): `octopus/tools/read_hijack.py:1-397` (units, arms, refusal
reasons, relation of R and S, the label set and its priority order, a resumable judge, the
mounted-vs-refused contrast with cluster-bootstrap intervals, judge precision on annotated
cases, a balanced export).
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
from dataclasses import dataclass, field
from pathlib import Path

from .cluster_boot import by_cluster, ci_text, contrast_ci, pooled_ci

# Label set in priority order (the judge gives the first that applies); results are keyed
# on these names.
LABELS = ("IDENTITY", "ROOT_CLOSE", "S_TASK", "OWN_USING_S", "OWN", "EMPTY", "UNCLEAR")
HIJACK = frozenset({"S_TASK", "IDENTITY"})
INVALID = ("ERROR", "UNPARSED", "UNLABELLED")
REASONS = ("not_readable_yet", "self", "other")
MOUNTED = re.compile(r"read_thread: mounted (\S+) steps (\d+)-(\d+) \((\d+) tokens\)")

JUDGE_PROMPT = """Classify one step of a multi-thread research agent.

How the agent works: the thread "main" owns the root question below and may split off sub-tasks to branch \
threads. A branch must stay on its own sub-task and close with a result for that sub-task; answering the root \
question is main's job alone. Every thread can call read_thread to look at another thread's steps.

Root question:
{question}

All threads and their sub-tasks:
{threads}

The step to classify was taken by branch {R} ("R"). R's own sub-task: {R_task}
Right before this step, R read thread {S} ("S"). S's sub-task: {S_task}

R's step (its text, then any tool calls):
<action>
{action}
</action>

Labels, checked in this order (pick the first one that fits):
IDENTITY - R speaks of S's steps as its own earlier work (e.g. "my search" for a search S ran), or acts as main \
(claims to be main, re-plans the whole job, or answers the whole root question).
ROOT_CLOSE - R closes its branch with an answer to the root question rather than its sub-task's result.
S_TASK - R works on S's sub-task (or some other thread's) rather than its own.
OWN_USING_S - R works on its own sub-task and uses facts, documents or results it got from S.
OWN - R works on its own sub-task.
EMPTY - neither a tool call nor any substantive text.
UNCLEAR - none of the above can be decided.
Answer with the label only."""


# ---------------------------------------------------------------------------- extraction
def reason(result: str) -> str:
    """What one read_thread result was: mounted, close_now, or a refusal reason."""
    from ..runtime.core import CLIPPED, RESERVE_NOTE

    if MOUNTED.match(result):
        return "mounted"
    reserve_head = RESERVE_NOTE.split("(")[0]
    if result.startswith(reserve_head) or CLIPPED in result:
        return "close_now"
    if "never itself" in result:
        return "self"
    if "has no readable step yet" in result:
        return "not_readable_yet"
    return "other"


def as_action(content: str | None, calls: list[str]) -> str:
    """One text form for logged and freshly sampled replies: the reply text, then one
    line per tool call."""
    text = (content or "").strip()
    if not calls:
        return text
    listing = "Tool calls:\n" + "\n".join(calls)
    return f"{text}\n{listing}" if text else listing


def action_text(msg: dict) -> str:
    fns = [c.get("function") or {} for c in msg.get("tool_calls") or []]
    return as_action(msg.get("content"), [f"{f.get('name')}({f.get('arguments')})" for f in fns])


def branches(tree: dict) -> dict:
    """Thread name -> (fork record, branch record), for branches at every depth."""
    from ..runtime.core import tree_branches

    return {name: (fork, rec) for name, fork, rec in tree_branches(tree.get("forks") or [])}


def relation(r: str, s: str | None) -> str:
    """How thread S sits relative to R in the thread tree."""
    if s is None:
        return "unknown"
    if s == r:
        return "self"
    if s == "main" or r.startswith(s + "/"):
        return "ancestor"
    if s.startswith(r + "/"):
        return "descendant"
    parent = lambda name: name.rsplit("/", 1)[0]  # noqa: E731
    return "sibling" if parent(s) == parent(r) else "cousin"


def resolve(name, names) -> str | None:
    """A requested thread as read_thread resolves it: "main", a full thread name, or a
    branch id that exactly one thread ends with."""
    if not isinstance(name, str):
        return None
    name = name.strip()
    if name == "main" or name in names:
        return name
    matches = [n for n in names if n.rsplit("/", 1)[-1] == name]
    return matches[0] if len(matches) == 1 else None


def cluster_of(run: str, question: str) -> str:
    return f"{run}/{hashlib.sha1(question.encode()).hexdigest()[:12]}"


@dataclass
class _Read:
    reply: int        # message index of the reply that issued the read
    requested: object
    result: str

    @property
    def kind(self) -> str:
        return reason(self.result)


@dataclass
class _Stretch:
    """Reads of a stretch of read/fork-only replies, and the substantive reply after it."""

    reads: list[_Read]
    action_index: int   # message index of the action reply
    reply_number: int   # 1-based among the branch's own replies
    own_replies: int


def _stretches(msgs: list[dict], first_own: int):
    """Walk a branch's own replies; yield a _Stretch for every substantive reply preceded
    by reads.  A substantive reply's own reads open the next stretch (they mount from the
    following reply on).  Returns whether reads were left without an action."""
    from ..runtime.core import decode_tool_call

    results = {m.get("tool_call_id"): str(m.get("content") or "") for m in msgs if m.get("role") == "tool"}
    own = [i for i in range(first_own, len(msgs)) if msgs[i].get("role") == "assistant"]
    carried: list[_Read] = []
    for number, i in enumerate(own, 1):
        calls = [decode_tool_call(c) for c in msgs[i].get("tool_calls") or []]
        reads = [_Read(i, args.get("thread"), results.get(cid, "")) for name, args, cid in calls
                 if name == "read_thread"]
        only_reads_or_forks = bool(calls) and all(name in ("read_thread", "fork") for name, _, _ in calls)
        if only_reads_or_forks:
            carried.extend(reads)
            continue
        if carried:
            yield _Stretch(carried, i, number, len(own))
        carried = reads
    return bool(carried)


def _unit(stretch: _Stretch, r_name: str, threads: dict, msgs: list[dict], ctx: dict) -> dict:
    kinds = [rd.kind for rd in stretch.reads]
    if "mounted" in kinds:
        last = max(k for k, kind in enumerate(kinds) if kind == "mounted")
        m = MOUNTED.match(stretch.reads[last].result)
        s_name, arm, refusal = m.group(1), "mounted", None
        read_reply, steps = stretch.reads[last].reply, [int(m.group(g)) for g in (2, 3, 4)]
    else:
        pick = next((k for k, rd in enumerate(stretch.reads) if resolve(rd.requested, threads)), 0)
        s_name = resolve(stretch.reads[pick].requested, threads)
        arm = "close_now" if "close_now" in kinds else "refused"
        refusal = kinds[pick] if arm == "refused" else None
        read_reply, steps = None, None
    tasks = ctx["tasks"]
    question = ctx["question"]
    return {
        "id": f"{ctx['run']}/{ctx['ep']}/{r_name}/{stretch.action_index}",
        "run": ctx["run"], "ep": ctx["ep"], "tree": ctx["tree"], "cluster": cluster_of(ctx["run"], question),
        "R": r_name, "S": s_name or str(stretch.reads[0].requested), "relation": relation(r_name, s_name),
        "arm": arm, "refusal": refusal, "mounted_before": ctx["mounted_before"], "read_reply": read_reply,
        "steps": steps, "reply_index": stretch.reply_number,
        "position": stretch.reply_number / stretch.own_replies,
        "read": " | ".join(rd.result.strip().split("\n", 1)[0][:200] for rd in stretch.reads),
        "question": question, "threads": tasks, "R_task": tasks[r_name],
        "S_task": question if s_name == "main" else tasks.get(s_name, "(no such thread)"),
        "action": action_text(msgs[stretch.action_index]),
    }


def tree_units(tree: dict, where: dict, stats: collections.Counter):
    """The units of one episode tree (`where`: run, ep, tree path)."""
    threads = branches(tree)
    question = tree.get("task") or next(
        (m["content"] for m in tree.get("main") or [] if m.get("role") == "user"), "")
    tasks = {name: rec.get("task") or "" for name, (_, rec) in threads.items()}
    for r_name, (_, rec) in threads.items():
        msgs = rec.get("messages")
        if msgs is None:
            stats["branch_without_history"] += 1
            continue
        ctx = {**where, "question": question, "tasks": tasks, "mounted_before": False}
        walk = _stretches(msgs, rec.get("prefix_len", 0))
        while True:
            try:
                stretch = next(walk)
            except StopIteration as end:
                stats["no_action_after_reads"] += bool(end.value)
                break
            unit = _unit(stretch, r_name, threads, msgs, ctx)
            stats[f"{unit['arm']}/{unit['refusal'] or ''}/{unit['relation']}"] += 1
            yield unit
            ctx["mounted_before"] = ctx["mounted_before"] or unit["arm"] == "mounted"


def extract_units(log_dirs) -> tuple[list[dict], collections.Counter]:
    stats, units = collections.Counter(), []
    for d in log_dirs:
        base = Path(d)
        for path in sorted(base.rglob("tree.json")):
            try:
                tree = json.loads(path.read_text())
            except (OSError, json.JSONDecodeError):
                stats["unreadable_tree"] += 1
                continue
            ep = path.parent.name if path.parent == base else str(path.parent.relative_to(base))
            units.extend(tree_units(tree, {"run": base.name, "ep": ep, "tree": str(path)}, stats))
    return units, stats


# ---------------------------------------------------------------------------- judging
def prompt(item: dict) -> str:
    listing = "\n".join(["main: the root question"] + [f"{n}: {t}" for n, t in item["threads"].items()])
    return JUDGE_PROMPT.format(threads=listing, **{k: item[k] for k in ("question", "R", "R_task", "S", "S_task",
                                                                        "action")})


_LABEL_RE = re.compile(r"\b(" + "|".join(sorted(LABELS, key=len, reverse=True)) + r")\b")


def parse(text: str) -> str:
    m = _LABEL_RE.search(text.upper())
    return m.group(1) if m else "UNPARSED"


def labels(path) -> dict:
    """id -> label; when an id appears twice, its later row wins (resumed runs append)."""
    p = Path(path)
    out = {}
    if p.exists():
        for line in p.read_text().splitlines():
            if line.strip():
                row = json.loads(line)
                out[row["id"]] = row["label"]
    return out


def http_post(url: str):
    """A judge client for an OpenAI-compatible /chat/completions endpoint."""
    endpoint = url.rstrip("/") + "/chat/completions"

    def post(body: dict) -> str:
        req = urllib.request.Request(endpoint, json.dumps(body).encode(), {"Content-Type": "application/json"})
        with urllib.request.urlopen(req, timeout=300) as resp:
            return json.load(resp)["choices"][0]["message"]["content"] or ""
    return post


def _label_one(item: dict, post, model: str, attempts: int = 3) -> dict:
    body = {"model": model, "temperature": 0, "max_tokens": 16, "chat_template_kwargs": {"enable_thinking": False},
            "messages": [{"role": "user", "content": prompt(item)}]}
    last = ""
    for _ in range(attempts):
        try:
            raw = post(body)
        except Exception as e:  # noqa: BLE001  (a judge failure becomes an ERROR row, not a crash)
            last = repr(e)[:200]
            continue
        return {"id": item["id"], "label": parse(raw), "raw": raw[:100]}
    return {"id": item["id"], "label": "ERROR", "raw": last}


def judge(items_path, labels_path, post, model: str = "judge", workers: int = 8) -> int:
    """Label every item that has no valid label yet, appending rows as they finish (a
    stopped run resumes where it stopped).  Returns 1 while invalid labels remain."""
    have = {i for i, lab in labels(labels_path).items() if lab not in INVALID}
    todo = [it for it in map(json.loads, Path(items_path).read_text().splitlines()) if it["id"] not in have]
    with open(labels_path, "a") as sink, cf.ThreadPoolExecutor(max(1, workers)) as pool:
        for row in pool.map(lambda it: _label_one(it, post, model), todo):
            sink.write(json.dumps(row) + "\n")
            sink.flush()
    left = collections.Counter(lab for lab in labels(labels_path).values() if lab in INVALID)
    print(f"labelled {len(todo)} items ({len(have)} before); invalid left: {dict(left)}")
    return 1 if left else 0


# ---------------------------------------------------------------------------- statistics
def boot(groups: list[list[float]], reps: int = 2000, seed: int = 0) -> tuple[float, float, float]:
    """Pooled mean of grouped values with a 95% interval resampling whole groups."""
    return pooled_ci(groups, reps, seed)


def boot_diff(rows: list[dict], f, arm, reps: int = 2000, seed: int = 0) -> tuple[float, float, float]:
    """Mean of f over rows with arm(row) minus over the rest; 95% interval over clusters."""
    return contrast_ci(rows, f, arm, reps, seed)


def rate(rows: list[dict], f) -> tuple[float, float, float]:
    return pooled_ci(by_cluster(rows, f))


fmt = ci_text


def mix(rows: list[dict]) -> str:
    if not rows:
        return "-"
    c = collections.Counter(u["label"] for u in rows)
    return " ".join(f"{k} {c[k] / len(rows):.2f}" for k in LABELS if c[k])


def load(units_path, labels_path) -> list[dict]:
    lab = labels(labels_path)
    return [{**u, "label": lab.get(u["id"], "UNLABELLED")} for u in map(json.loads,
                                                                         Path(units_path).read_text().splitlines())]


@dataclass
class _Table:
    head: list[str]
    out: object
    rows: list = field(default_factory=list)

    def __post_init__(self):
        self.out("| " + " | ".join(self.head) + " |")
        self.out("|" + "---|" * len(self.head))

    def row(self, *cells):
        self.out("| " + " | ".join(str(c) for c in cells) + " |")


def _is_hijack(u):
    return u["label"] in HIJACK


def _is_root_close(u):
    return u["label"] == "ROOT_CLOSE"


def _is_mounted(u):
    return u["arm"] == "mounted"


def report(units_path, labels_path, annotated=None, out=print) -> int:
    rows = load(units_path, labels_path)
    invalid = collections.Counter(u["label"] for u in rows if u["label"] in INVALID)
    out(f"invalid labels left out of every rate: {dict(invalid) or 'none'}")
    rows = [u for u in rows if u["label"] not in INVALID]
    out(f"{len(rows)} labelled units, {len({u['cluster'] for u in rows})} question groups; hijack = S_TASK or "
        "IDENTITY; position = reply index / R's own replies; 95% bootstrap CIs over question groups\n")
    runs = sorted({u["run"] for u in rows})
    groups = [("all", lambda u: True), ("no earlier mount", lambda u: not u["mounted_before"])]
    groups += [(rel, lambda u, rel=rel: u["relation"] == rel)
               for rel in ("sibling", "cousin", "descendant", "ancestor", "self", "unknown")]
    t = _Table(["run", "group", "mounted / refused", "hijack mounted", "hijack refused", "mounted - refused",
                "ROOT_CLOSE mounted - refused", "position mounted - refused"], out)
    for run in runs:
        for name, sel in groups:
            sub = [u for u in rows if u["run"] == run and u["arm"] != "close_now" and sel(u)]
            if not sub:
                continue
            mounted = [u for u in sub if _is_mounted(u)]
            refused = [u for u in sub if not _is_mounted(u)]
            t.row(run, name, f"{len(mounted)} / {len(refused)}", fmt(rate(mounted, _is_hijack)) if mounted else "-",
                  fmt(rate(refused, _is_hijack)) if refused else "-", fmt(boot_diff(sub, _is_hijack, _is_mounted)),
                  fmt(boot_diff(sub, _is_root_close, _is_mounted)),
                  fmt(boot_diff(sub, lambda u: u["position"], _is_mounted)))
    out("")
    arms = [("mounted", _is_mounted)] + [(f"refused: {x}", lambda u, x=x: u["refusal"] == x) for x in REASONS]
    arms.append(("close_now", lambda u: u["arm"] == "close_now"))
    t = _Table(["run", "arm", "n", "hijack", "ROOT_CLOSE", "position", "reply index", "labels"], out)
    for run in runs:
        for name, sel in arms:
            sub = [u for u in rows if u["run"] == run and sel(u)]
            if sub:
                t.row(run, name, len(sub), fmt(rate(sub, _is_hijack)), fmt(rate(sub, _is_root_close)),
                      fmt(rate(sub, lambda u: u["position"])), fmt(rate(sub, lambda u: u["reply_index"])), mix(sub))
    if annotated:
        precision(rows, annotated, out)
    if invalid:
        out(f"\nNO RESULT: {sum(invalid.values())} units have no valid label; rerun judge")
        return 1
    return 0


def precision(rows: list[dict], annotated, out=print) -> dict:
    """Per-label precision of the judge against hand-annotated cases (export's file with
    the label column filled in), plus hijack precision and recall."""
    judged = {u["id"]: u["label"] for u in rows}
    cases = [c for c in map(json.loads, Path(annotated).read_text().splitlines())
             if c["id"] in judged and c.get("label")]
    annotators = sorted({c.get("annotator", "") for c in cases})
    out(f"\njudge vs annotated labels ({', '.join(annotators)}) on {len(cases)} cases\n")
    t = _Table(["judge label", "n", "precision"], out)
    res = {}
    for lab in LABELS:
        hits = [c["label"] == lab for c in cases if judged[c["id"]] == lab]
        if hits:
            res[lab] = sum(hits) / len(hits)
            t.row(lab, len(hits), f"{res[lab]:.2f}")
    said = [c for c in cases if judged[c["id"]] in HIJACK]
    truth = [c for c in cases if c["label"] in HIJACK]
    res["hijack_precision"] = sum(c["label"] in HIJACK for c in said) / max(1, len(said))
    res["hijack_recall"] = sum(judged[c["id"]] in HIJACK for c in truth) / max(1, len(truth))
    t.row("hijack", len(said), f"{res['hijack_precision']:.2f} (recall {res['hijack_recall']:.2f} of {len(truth)})")
    return res


def export(units_path, cases_path, n: int = 120) -> int:
    """Up to n units to annotate by hand, half mounted and half refused (seed 0), carrying
    only the judge's inputs (the arm is withheld so the annotator is blind to it)."""
    units = list(map(json.loads, Path(units_path).read_text().splitlines()))
    rng = random.Random(0)
    picked = []
    for arm in ("mounted", "refused"):
        pool = [u for u in units if u["arm"] == arm]
        picked.extend(rng.sample(pool, min(len(pool), n // 2)))
    rng.shuffle(picked)
    fields = ("id", "question", "threads", "R", "R_task", "S", "S_task", "action")
    with open(cases_path, "w") as f:
        for u in picked:
            f.write(json.dumps({**{k: u[k] for k in fields}, "label": "", "annotator": ""}, ensure_ascii=False) + "\n")
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
            f.writelines(json.dumps(u, ensure_ascii=False) + "\n" for u in units)
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
