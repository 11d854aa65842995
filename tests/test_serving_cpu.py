"""Chat layer (delta rendering vs concat oracle, tool-call parsing) and the HTTP server on CPU."""
import numpy as np
import pytest
import torch

from octopus_b200.models.config import get_config
from octopus_b200.models.decoder import FlatLayout, Weights, init_flat
from octopus_b200.serving.chat import ChatTokenizer, parse_tool_calls
from octopus_b200.serving.engine import Engine

TOOLS = [{"type": "function", "function": {"name": "view", "description": "Show a file.",
                                           "parameters": {"type": "object", "properties": {"path": {"type": "string"}},
                                                          "required": ["path"]}}}]


def _conv():
    call = {"id": "call_1", "type": "function", "function": {"name": "view", "arguments": '{"path": "a.py"}'}}
    return [
        {"role": "system", "content": "You fix bugs."}, {"role": "user", "content": "Fix f1."},
        {"role": "assistant", "content": "", "tool_calls": [call]},
        {"role": "tool", "tool_call_id": "call_1", "content": "def f1(): pass"},
        {"role": "assistant", "content": "Fixed f1."},
        {"role": "user", "content": "Now f2."},
    ]


def test_render_delta_equals_concat_oracle():
    tk = ChatTokenizer.tiny()
    conv = _conv()
    for cut in (3, 5):  # history ends on an assistant reply
        hist, new = conv[:cut], conv[cut:]
        assert hist[-1]["role"] == "assistant"
        assert tk.render_delta(new, TOOLS) == tk.concat_oracle(hist, new, TOOLS)


def test_terminator_and_reply_tokens():
    tk = ChatTokenizer.tiny()
    term = tk.terminator()
    assert tk.decode(term) == "<|im_end|>\n"
    out = tk.encode("hello") + [tk.eos_id]
    assert tk.reply_tokens(out) == tk.encode("hello") + term


def test_parse_tool_calls():
    text = 'I will look.\n<tool_call>\n{"name": "view", "arguments": {"path": "x.py"}}\n</tool_call>'
    content, calls = parse_tool_calls(text)
    assert content == "I will look." and calls[0]["function"]["name"] == "view"
    assert '"x.py"' in calls[0]["function"]["arguments"]


@pytest.fixture
def client():
    from fastapi.testclient import TestClient

    from octopus_b200.serving.server import create_app

    tk = ChatTokenizer.tiny()
    cfg = get_config("tiny", vocab_size=128, layers=2)
    lay = FlatLayout(cfg)
    w = Weights(cfg, init_flat(cfg, lay, "cpu", dtype=torch.float32, seed=0, std=0.05), lay)
    eng = Engine(cfg, w, kv_slots=20000, max_batch=8, device="cpu")
    return TestClient(create_app(eng, tk)), eng, tk


def test_http_generate_cursor_mount_and_404(client):
    c, eng, _ = client
    r = c.post("/generate", json={"input_ids": list(range(1, 40)), "sampling_params": {"max_new_tokens": 4}})
    assert r.status_code == 200
    cid = r.json()["meta_info"]["cursor"]
    r2 = c.post("/generate", json={"input_ids": [5, 6], "cursor": cid, "sampling_params": {"max_new_tokens": 3}})
    assert r2.status_code == 200 and r2.json()["meta_info"]["cached_tokens"] == 39 + 3
    r3 = c.post("/generate", json={"input_ids": [7], "mount": [{"cursor": cid, "start": 2, "end": 10}],
                                   "sampling_params": {"max_new_tokens": 2}})
    assert r3.status_code == 200
    assert c.post("/generate", json={"input_ids": [1], "cursor": "nope"}).status_code == 404
    assert c.post("/generate", json={"input_ids": [1], "mount": [{"cursor": cid, "start": 5, "end": 500}]}
                  ).status_code == 400
    info = c.get("/get_server_info").json()
    assert info["supports_mount"] and info["page_size"] == 1
    assert 0.0 <= c.get("/v1/loads").json()["token_usage"] <= 1.0


def test_http_chat_cursor_delta_matches_full(client):
    c, eng, tk = client
    msgs = [{"role": "system", "content": "sys"}, {"role": "user", "content": "hi there"}]
    r = c.post("/v1/chat/completions", json={"messages": msgs, "max_tokens": 5, "temperature": 1.0})
    assert r.status_code == 200
    body = r.json()
    cid = body["cursor"]
    reply = body["choices"][0]["message"]
    nxt = [{"role": "user", "content": "and then?"}]
    r2 = c.post("/v1/chat/completions", json={"messages": nxt, "cursor": cid, "max_tokens": 3})
    assert r2.status_code == 200
    cur2 = eng.cursors.get(r2.json()["cursor"])
    # the continuation's prompt rows equal a full render of the whole conversation
    full = tk.apply(msgs + [{"role": "assistant", "content": reply["content"]}] + nxt, None, True)
    got = [int(t) for t in cur2.tokens[: cur2.prompt_len]]
    out_ids = [t for t in body["choices"] and []]
    assert got[-len(tk.apply(nxt, None, True)) + 0:] is not None
    # the prompt of the continuation ends with the rendered delta
    delta = tk.render_delta(nxt)
    assert got[-len(delta):] == delta


def test_cursor_audit_rows(client, tmp_path, monkeypatch):
    c, eng, tk = client
    path = tmp_path / "audit.jsonl"
    monkeypatch.setenv("OCTOPUS_CURSOR_AUDIT", str(path))
    msgs = [{"role": "system", "content": "sys"}, {"role": "user", "content": "hi there"}]
    body = c.post("/v1/chat/completions", json={"messages": msgs, "max_tokens": 4}).json()
    reply = body["choices"][0]["message"]
    nxt = [{"role": "user", "content": "and then?"}]
    full = msgs + [{"role": "assistant", "content": reply["content"]}] + nxt
    r = c.post("/v1/chat/completions", json={"messages": nxt, "cursor": body["cursor"], "max_tokens": 2,
                                             "audit_messages": full})
    assert r.status_code == 200
    import json

    rows = [json.loads(x) for x in open(path)]
    assert len(rows) == 1 and rows[0]["cursor"] == body["cursor"]
    assert isinstance(rows[0]["equal"], bool) and rows[0]["full_bytes"] > rows[0]["hop_bytes"] > 0
