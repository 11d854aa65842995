"""Token ids and loss labels of a fork tree.

A chat template may render a turn differently once later messages follow it, so the
root is never rendered on its own: each child is rendered together with the root, and
the joint text is split where the child's first message block begins (the block marker
that follows the root's last block).  All children must yield the very same root text;
otherwise the tree is dropped.  A token is labelled (trained) when it lies inside an
assistant reply, i.e. after an assistant block header up to and including its
end-of-turn marker; every other token gets IGNORE.  Children are always labelled; the
root only in a tree with ``train_root``.

Reference parity (behaviour): `octopus/tools/tree_sft/encode.py:1-104` (joint rendering
with the root split off, exact-root check, assistant-span labels, whole-tree drops, flat
rows whose join row carries the root's labels).
"""
from __future__ import annotations

import bisect
import json
import re

IGNORE = -100
BLOCK = "<|im_start|>"
_BLOCK_RE = re.compile(re.escape(BLOCK))
_REPLY_RE = re.compile(r"<\|im_start\|>assistant\n(.*?<\|im_end\|>)", re.S)


def _mapping(arguments) -> dict:
    """Tool-call arguments as a mapping (wire logs hold JSON strings)."""
    if isinstance(arguments, dict):
        return arguments
    try:
        parsed = json.loads(arguments or "{}")
    except (TypeError, json.JSONDecodeError):
        return {"raw": str(arguments)}
    return parsed if isinstance(parsed, dict) else {"raw": parsed}


def for_template(msg: dict) -> dict:
    """A logged OpenAI-wire message in the form chat templates expect: string content
    and tool-call arguments as mappings."""
    calls = msg.get("tool_calls")
    out = {**msg, "content": msg.get("content") or ""}
    if calls:
        out["tool_calls"] = [
            {**c, "function": {**c["function"], "arguments": _mapping(c["function"].get("arguments"))}} for c in calls]
    return out


def render(tok, messages: list[dict], tools) -> str:
    return tok.render([for_template(m) for m in messages], tools, False)


class _ReplySpans:
    """Character spans of assistant replies in one text, for token labelling."""

    def __init__(self, text: str):
        spans = [m.span(1) for m in _REPLY_RE.finditer(text)]
        self.starts = [s for s, _ in spans]
        self.ends = [e for _, e in spans]

    def covers(self, a: int, b: int) -> bool:
        """True if characters [a, b) lie within one reply span."""
        k = bisect.bisect_right(self.starts, a) - 1
        return k >= 0 and b <= self.ends[k]


def labelled_ids(tok, text: str) -> tuple[list[int], list[int]]:
    """(ids, labels) of `text`: labels[i] = ids[i] for tokens inside assistant replies."""
    enc = tok.tok.encode(text, add_special_tokens=False)
    spans = _ReplySpans(text)
    ids = list(enc.ids)
    labels = [tid if spans.covers(a, b) else IGNORE for tid, (a, b) in zip(ids, enc.offsets)]
    return ids, labels


def _split_at_block(text: str, block_no: int) -> int:
    """Character offset of the `block_no`-th (0-based) message block marker in `text`."""
    for k, m in enumerate(_BLOCK_RE.finditer(text)):
        if k == block_no:
            return m.start()
    raise ValueError(f"rendered text has no block number {block_no}")


def encode_tree(tree: dict, tok, max_len: int, min_child_tokens: int = 256,
                max_tree_tokens: int | None = None) -> dict | None:
    """{root_ids, root_labels, children: [{kind, ids, labels}]} or None (tree dropped).

    A tree is dropped whole, never truncated (no child may lose its closing turns), when
    the root text differs between children, when root plus some child exceeds max_len
    or leaves less than min_child_tokens of room, when no child has a labelled token, or
    when root plus all children exceed max_tree_tokens."""
    tools, root = tree.get("tools"), tree["root"]
    first_child_block = len(_BLOCK_RE.findall(render(tok, root, tools)))
    root_texts, children = set(), []
    for child in tree["children"]:
        joint = render(tok, root + child["messages"], tools)
        at = _split_at_block(joint, first_child_block)
        root_texts.add(joint[:at])
        ids, labels = labelled_ids(tok, joint[at:])
        children.append({"kind": child["kind"], "ids": ids, "labels": labels})
    if len(root_texts) != 1:  # no child, or children that disagree on the root
        return None
    root_ids, root_labels = labelled_ids(tok, root_texts.pop())
    if not tree.get("train_root"):
        root_labels = [IGNORE] * len(root_ids)
    room = max_len - len(root_ids)
    if room < min_child_tokens or max(len(c["ids"]) for c in children) > room:
        return None
    children = [c for c in children if any(x != IGNORE for x in c["labels"])]
    total = len(root_ids) + sum(len(c["ids"]) for c in children)
    if not children or (max_tree_tokens and total > max_tree_tokens):
        return None
    return {"root_ids": root_ids, "root_labels": root_labels, "children": children}


def flat_rows(enc: dict) -> list[dict]:
    """The tree as independent sequences (root + one child each).  The root's labels go
    to the join child's row only (the first child if there is none), so each token is
    trained exactly once, as in the tree form."""
    root = enc["root_ids"]
    silent = [IGNORE] * len(root)
    root_labels = enc.get("root_labels") or silent
    kinds = [c["kind"] for c in enc["children"]]
    owner = kinds.index("join") if "join" in kinds else 0
    return [{"input_ids": root + c["ids"], "labels": (root_labels if k == owner else silent) + c["labels"],
             "kind": c["kind"]} for k, c in enumerate(enc["children"])]
