"""Fork trees as token ids with per-token loss labels.

Each child is rendered together with the root (a template may format earlier turns
differently once later messages exist), and the root is cut out of that joint rendering at
the turn marker where the child starts; every child must give the exact same root text, or
the tree is dropped.  Labels are the ids of tokens inside assistant blocks (the reply text
after the block header, through the end-of-turn marker) and IGNORE elsewhere: in every
child, and in the root only for a tree with `train_root`.

Reference parity (behaviour): `octopus/tools/tree_sft/encode.py:1-104` (joint rendering and
root cut, exact-root check, assistant-span labels, whole-tree drops, flat rows with the
root's labels carried by the join row).
"""
from __future__ import annotations

import json
import re

IGNORE = -100
BLOCK = "<|im_start|>"
ASSISTANT = re.compile(r"<\|im_start\|>assistant\n(.*?<\|im_end\|>)", re.S)


def _arguments(raw) -> dict:
    if isinstance(raw, dict):
        return raw
    try:
        v = json.loads(raw or "{}")
    except (TypeError, json.JSONDecodeError):
        return {"raw": str(raw)}
    return v if isinstance(v, dict) else {"raw": v}


def for_template(m: dict) -> dict:
    """Logged (OpenAI wire) messages for a chat template: string content, argument mappings."""
    out = dict(m)
    out["content"] = out.get("content") or ""
    if out.get("tool_calls"):
        out["tool_calls"] = [{**c, "function": {**c["function"], "arguments": _arguments(c["function"].get("arguments"))}}
                             for c in out["tool_calls"]]
    return out


def render(tok, messages: list[dict], tools) -> str:
    return tok.render([for_template(m) for m in messages], tools, False)


def _cut(text: str, n_blocks: int) -> int:
    pos = -1
    for _ in range(n_blocks + 1):
        pos = text.index(BLOCK, pos + 1)
    return pos


def labelled_ids(tok, text: str) -> tuple[list[int], list[int]]:
    enc = tok.tok.encode(text, add_special_tokens=False)
    spans = [m.span(1) for m in ASSISTANT.finditer(text)]
    labels = [tid if any(s <= a and b <= e for s, e in spans) else IGNORE
              for tid, (a, b) in zip(enc.ids, enc.offsets)]
    return list(enc.ids), labels


def encode_tree(tree: dict, tok, max_len: int, min_child_tokens: int = 256,
                max_tree_tokens: int | None = None) -> dict | None:
    """{root_ids, root_labels, children: [{kind, ids, labels}]}, or None when the root is not
    shared exactly, root + a child exceeds max_len (trees are dropped whole, never cut, so
    no child loses its closing turns), or root + all children exceed max_tree_tokens."""
    tools, root = tree.get("tools"), tree["root"]
    n_root = render(tok, root, tools).count(BLOCK)
    root_text, children = None, []
    for child in tree["children"]:
        full = render(tok, root + child["messages"], tools)
        cut = _cut(full, n_root)
        if root_text is None:
            root_text = full[:cut]
        elif full[:cut] != root_text:
            return None
        ids, labels = labelled_ids(tok, full[cut:])
        children.append({"kind": child["kind"], "ids": ids, "labels": labels})
    root_ids, root_labels = labelled_ids(tok, root_text)
    if not tree.get("train_root"):
        root_labels = [IGNORE] * len(root_ids)
    room = max_len - len(root_ids)
    if room < min_child_tokens or any(len(c["ids"]) > room for c in children):
        return None
    children = [c for c in children if any(x != IGNORE for x in c["labels"])]
    if not children:
        return None
    if max_tree_tokens and len(root_ids) + sum(len(c["ids"]) for c in children) > max_tree_tokens:
        return None
    return {"root_ids": root_ids, "root_labels": root_labels, "children": children}


def flat_rows(enc: dict) -> list[dict]:
    """One sequence per child (root + child); the root's labels go into the join row only,
    so each token is trained once, as in the tree form."""
    root = enc["root_ids"]
    rl = enc.get("root_labels") or [IGNORE] * len(root)
    carrier = next((i for i, c in enumerate(enc["children"]) if c["kind"] == "join"), 0)
    return [{"input_ids": root + c["ids"], "labels": (rl if i == carrier else [IGNORE] * len(root)) + c["labels"],
             "kind": c["kind"]} for i, c in enumerate(enc["children"])]
