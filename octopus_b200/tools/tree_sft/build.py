"""Encode the fork trees of episode logs into a tree SFT dataset.

    python -m octopus_b200.tools.tree_sft.build --logs LOG_DIR [LOG_DIR ...] --out encoded.jsonl
        [--tokenizer HF_DIR] [--max-len 65536] [--max-tree-tokens 131072] [--min-reward 1.0]

One line per tree: {task, trial, fork_no, root_ids, root_labels, children: [{kind, ids,
labels}]}; prints the counts that survived each filter.

Reference parity (behaviour): `octopus/tools/tree_sft/build.py:1-52`.
"""
from __future__ import annotations

import argparse
import collections
import json

from .encode import IGNORE, encode_tree
from .trees import collect


def build(log_dirs, tok, out_path, max_len: int = 65536, max_tree_tokens: int | None = 131072,
          min_reward: float | None = 1.0) -> dict:
    trees = collect(log_dirs, min_reward)
    stats = collections.Counter(trees=len(trees))
    with open(out_path, "w") as sink:
        for tree in trees:
            enc = encode_tree(tree, tok, max_len, max_tree_tokens=max_tree_tokens)
            if enc is None:
                stats["dropped"] += 1
                continue
            stats["kept"] += 1
            stats["children"] += len(enc["children"])
            stats["root_tokens"] += len(enc["root_ids"])
            stats["child_tokens"] += sum(len(c["ids"]) for c in enc["children"])
            stats["labelled_tokens"] += sum(sum(x != IGNORE for x in c["labels"]) for c in enc["children"]) + \
                sum(x != IGNORE for x in enc["root_labels"])
            sink.write(json.dumps({"task": tree["task"], "trial": tree["trial"], "fork_no": tree["fork_no"], **enc})
                       + "\n")
    return dict(stats)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m octopus_b200.tools.tree_sft.build")
    ap.add_argument("--logs", nargs="+", required=True)
    ap.add_argument("--out", required=True)
    ap.add_argument("--tokenizer", default="", help="HF tokenizer directory (default: the built-in tiny one)")
    ap.add_argument("--max-len", type=int, default=65536, help="root + one child")
    ap.add_argument("--max-tree-tokens", type=int, default=131072, help="root + all children")
    ap.add_argument("--min-reward", type=float, default=1.0)
    args = ap.parse_args(argv)
    from ...serving.chat import ChatTokenizer

    tok = ChatTokenizer.from_dir(args.tokenizer) if args.tokenizer else ChatTokenizer.tiny()
    print(json.dumps(build(args.logs, tok, args.out, args.max_len, args.max_tree_tokens, args.min_reward)))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
