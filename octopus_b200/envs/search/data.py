"""Questions for the search environment, read from downloaded Hugging Face parquet files at
run time (only question ids belong in a repository).

- OpenResearcher (train / validation): the Gold-Doc corpus's questions with their pass
  rates.  `split` writes a deterministic ids-only split (seed 0, stratified by pass rate in
  1/16 bins: 500 validation questions, then 3,040 train questions from the rest); `export`
  writes the RL inputs (questions.jsonl {qid, question, answer}, train-qids.txt,
  validation-qids.txt).  Answers wrapped as `\\boxed{...}` are unwrapped.
- BrowseComp-Plus (test): 830 queries whose fields are obfuscated in the published files
  (base64 of the text XOR-ed with the SHA-256 digest of the canary line in the dataset
  README).  `browsecomp_plus()` decodes them in memory only; its output must not be written
  into a repository or committed logs.

    python -m octopus_b200.envs.search.data split GOLD_DOC_DIR --out split.json
    python -m octopus_b200.envs.search.data export GOLD_DOC_DIR OUT_DIR [--split split.json]

Reference parity (behaviour): `octopus/envs/search/data.py:1-97` (unboxing, the stratified
largest-remainder split, the export files, the BrowseComp-Plus field decoding).
"""
from __future__ import annotations

import argparse
import base64
import collections
import glob
import hashlib
import json
import os
import random
import re


def _parquet(dataset_dir: str, columns: list[str]) -> list[dict]:
    import pyarrow.parquet as pq

    rows = []
    for f in sorted(glob.glob(os.path.join(dataset_dir, "data", "*.parquet"))):
        rows += pq.read_table(f, columns=columns).to_pylist()
    return rows


_BOXED = re.compile(r"\s*(\$*)\s*\\boxed\{(.*)\}\s*\1\s*", re.S)


def unbox(answer: str) -> str:
    """`\\boxed{x}` (alone or inside $ / $$) -> x, with `\\text{y}` -> y; anything else unchanged
    (also a boxed answer whose brace closes early: `\\boxed{a} and \\boxed{b}`)."""
    m = _BOXED.fullmatch(answer)
    if not m:
        return answer
    depth = 0
    for ch in m.group(2):
        depth += (ch == "{") - (ch == "}")
        if depth < 0:
            return answer
    if depth:
        return answer
    inner = re.sub(r"\\text\{([^{}]*)\}", r"\1", m.group(2))
    return re.sub(r" {2,}", " ", inner).strip()


def openresearcher(dataset_dir: str) -> dict:
    """query_id -> {query_id, query, answer (unboxed), pass_rate}."""
    return {r["query_id"]: {**r, "answer": unbox(r["answer"])}
            for r in _parquet(dataset_dir, ["query_id", "query", "answer", "pass_rate"])}


def allocate(sizes: dict, n: int) -> dict:
    """n split over strata in proportion to their sizes, largest remainders first (ties: the
    smaller stratum key)."""
    total = sum(sizes.values())
    n = min(n, total)  # (a smaller corpus than the split asks for: everything)
    if n <= 0:
        return {s: 0 for s in sizes}
    quota = {s: n * c / total for s, c in sizes.items()}
    out = {s: int(q) for s, q in quota.items()}
    for s in sorted(sizes, key=lambda s: (out[s] - quota[s], s))[: n - sum(out.values())]:
        out[s] += 1
    return out


def make_split(pass_rate: dict, n_val: int = 500, n_train: int = 3040, seed: int = 0) -> dict:
    """{qid: pass rate} -> {"validation": ids, "train": ids}, both stratified by pass rate in
    1/16 bins (a rate between bins goes to the nearest)."""
    rng = random.Random(seed)
    strata = collections.defaultdict(list)
    for q in sorted(pass_rate):
        strata[round(pass_rate[q] * 16)].append(q)
    for s in sorted(strata):
        rng.shuffle(strata[s])
    val = allocate({s: len(v) for s, v in strata.items()}, n_val)
    rest = {s: v[val[s]:] for s, v in strata.items()}
    train = allocate({s: len(v) for s, v in rest.items()}, n_train)
    return {"validation": sorted(q for s, v in strata.items() for q in v[: val[s]]),
            "train": sorted(q for s, v in rest.items() for q in v[: train[s]])}


def openresearcher_split(name: str, dataset_dir: str, split_path: str) -> list[dict]:
    """The questions of split `name` ("train" | "validation"), in split-file order."""
    rows = openresearcher(dataset_dir)
    with open(split_path) as f:
        return [rows[q] for q in json.load(f)[name]]


def _xor_key(canary: str) -> bytes:
    return hashlib.sha256(canary.encode()).digest()


def decode_field(text: str, canary: str) -> str:
    """A BrowseComp-Plus field: base64 bytes XOR-ed with the canary's SHA-256 digest (repeated)."""
    data, key = base64.b64decode(text), _xor_key(canary)
    return bytes(b ^ key[i % len(key)] for i, b in enumerate(data)).decode()


def encode_field(text: str, canary: str) -> str:
    """The inverse of decode_field (test fixtures)."""
    data, key = text.encode(), _xor_key(canary)
    return base64.b64encode(bytes(b ^ key[i % len(key)] for i, b in enumerate(data))).decode()


def canary(dataset_dir: str) -> str:
    """The canary line at the end of the dataset README (the decoding password)."""
    with open(os.path.join(dataset_dir, "README.md")) as f:
        found = re.findall(r"BENCHMARK DATA SHOULD NEVER APPEAR[^\n]*?browsecomp:[0-9a-f-]+", f.read())
    if not found:
        raise ValueError("no BrowseComp canary line in the dataset README")
    return found[-1]


def browsecomp_plus(dataset_dir: str) -> dict:
    """query_id -> {query_id, query, answer, evidence_docids, gold_docids}, decoded in memory."""
    pw, out = canary(dataset_dir), {}
    for r in _parquet(dataset_dir, ["query_id", "query", "answer", "evidence_docs", "gold_docs"]):
        out[r["query_id"]] = {"query_id": r["query_id"], "query": decode_field(r["query"], pw),
                              "answer": decode_field(r["answer"], pw),
                              "evidence_docids": [decode_field(d["docid"], pw) for d in r["evidence_docs"]],
                              "gold_docids": [decode_field(d["docid"], pw) for d in r["gold_docs"]]}
    return out


def export(dataset_dir: str, out_dir: str, split_path: str | None = None) -> dict:
    """questions.jsonl ({qid, question, answer}), train-qids.txt, validation-qids.txt."""
    rows = openresearcher(dataset_dir)
    if split_path:
        with open(split_path) as f:
            split = json.load(f)
    else:
        split = make_split({q: r["pass_rate"] for q, r in rows.items()})
    os.makedirs(out_dir, exist_ok=True)
    with open(os.path.join(out_dir, "questions.jsonl"), "w") as f:
        for q in sorted(rows):
            f.write(json.dumps({"qid": q, "question": rows[q]["query"], "answer": rows[q]["answer"]}) + "\n")
    for name in ("train", "validation"):
        with open(os.path.join(out_dir, f"{name}-qids.txt"), "w") as f:
            f.write("\n".join(str(q) for q in split[name]) + "\n")
    return {k: len(v) for k, v in split.items()}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m octopus_b200.envs.search.data")
    sub = ap.add_subparsers(dest="cmd", required=True)
    s = sub.add_parser("split")
    s.add_argument("dataset_dir")
    s.add_argument("--out", required=True)
    s.add_argument("--val", type=int, default=500)
    s.add_argument("--train", type=int, default=3040)
    e = sub.add_parser("export")
    e.add_argument("dataset_dir")
    e.add_argument("out_dir")
    e.add_argument("--split", default=None)
    args = ap.parse_args(argv)
    if args.cmd == "split":
        rows = openresearcher(args.dataset_dir)
        sp = make_split({q: r["pass_rate"] for q, r in rows.items()}, args.val, args.train)
        with open(args.out, "w") as f:
            json.dump(sp, f)
        print(json.dumps({k: len(v) for k, v in sp.items()}))
        return 0
    print(json.dumps(export(args.dataset_dir, args.out_dir, args.split)))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
