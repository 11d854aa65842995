"""Tool-call parsers on CPU: every format family yields OpenAI tool calls with the right
names and arguments and strips the markup from the content; qwen3_coder types parameters by
the tool schema; malformed calls stay text; the chat template picks the family; the chat
service uses it."""
import json

import pytest

from octopus_b200.serving.tool_parsers import detect_format, parse

TOOLS = [{"type": "function", "function": {"name": "view", "parameters": {"properties": {
    "path": {"type": "string"}, "start": {"type": "integer"}, "flags": {"type": "array"}}}}}]


def _args(calls):
    return [(c["function"]["name"], json.loads(c["function"]["arguments"])) for c in calls]


CASES = [
    ("qwen25", 'Look.\n<tool_call>\n{"name": "view", "arguments": {"path": "a.py"}}\n</tool_call>',
     [("view", {"path": "a.py"})]),
    ("hermes", '<tool_call>{"name": "view", "arguments": {"path": "a"}}</tool_call><tool_call>{"name": "done", '
     '"arguments": {}}</tool_call>', [("view", {"path": "a"}), ("done", {})]),
    ("qwen3_coder", "Look.\n<tool_call>\n<function=view>\n<parameter=path>\na.py\n</parameter>\n<parameter=start>\n12\n"
     "</parameter>\n<parameter=flags>\n[1, 2]\n</parameter>\n</function>\n</tool_call>",
     [("view", {"path": "a.py", "start": 12, "flags": [1, 2]})]),
    ("llama3", '<|python_tag|>{"name": "view", "parameters": {"path": "a"}}; {"name": "done", "parameters": {}}',
     [("view", {"path": "a"}), ("done", {})]),
    ("mistral", 'Look.[TOOL_CALLS][{"name": "view", "arguments": {"path": "a"}}]', [("view", {"path": "a"})]),
    ("mistral", 'Look.[TOOL_CALLS]view[ARGS]{"path": "a"}[TOOL_CALLS]done[ARGS]{}',
     [("view", {"path": "a"}), ("done", {})]),
    ("deepseekv3", "Look.<｜tool▁calls▁begin｜><｜tool▁call▁begin｜>function<｜tool▁sep｜>view\n```json\n"
     '{"path": "a"}\n```<｜tool▁call▁end｜><｜tool▁calls▁end｜>', [("view", {"path": "a"})]),
    ("deepseekv31", 'Look.<｜tool▁calls▁begin｜><｜tool▁call▁begin｜>view<｜tool▁sep｜>{"path": "a"}'
     "<｜tool▁call▁end｜><｜tool▁calls▁end｜>", [("view", {"path": "a"})]),
    ("glm45", "Look.<tool_call>view\n<arg_key>path</arg_key>\n<arg_value>a.py</arg_value>\n<arg_key>start</arg_key>\n"
     "<arg_value>3</arg_value>\n</tool_call>", [("view", {"path": "a.py", "start": 3})]),
    ("kimi_k2", 'Look.<|tool_calls_section_begin|><|tool_call_begin|>functions.view:0<|tool_call_argument_begin|>'
     '{"path": "a"}<|tool_call_end|><|tool_calls_section_end|>', [("view", {"path": "a"})]),
    ("gpt-oss", 'Look.<|start|>assistant<|channel|>commentary to=functions.view <|constrain|>json<|message|>'
     '{"path": "a"}<|call|>', [("view", {"path": "a"})]),
]


@pytest.mark.parametrize("fmt,text,want", CASES)
def test_formats(fmt, text, want):
    content, calls = parse(text, fmt, TOOLS)
    assert _args(calls) == want
    assert all(c["id"].startswith("call_") and c["type"] == "function" for c in calls)
    for marker in ("<tool_call>", "<function=", "[TOOL_CALLS]", "tool▁call", "<|tool_call", "<|call|>",
                   "<|python_tag|>"):
        assert marker not in content
    if text.startswith("Look."):
        assert content.startswith("Look.")


def test_malformed_and_plain_text():
    assert parse("no call here", "qwen3_coder") == ("no call here", [])
    bad = '<tool_call>{"name": "view", "arguments": {"path": }</tool_call>'
    assert parse(bad, "qwen25") == (bad, [])
    assert parse("just words", "llama3") == ("just words", [])
    with pytest.raises(ValueError):
        parse("x", "nope")


def test_detect_format():
    from octopus_b200.serving.chat import CHATML_TEMPLATE

    assert detect_format(CHATML_TEMPLATE) == "qwen25"
    assert detect_format("{{ '<tool_call>\\n<function=' + name }}") == "qwen3_coder"
    assert detect_format("<|python_tag|>") == "llama3" and detect_format(None) == "qwen25"
    assert detect_format("<｜tool▁call▁begin｜>function<｜tool▁sep｜>") == "deepseekv3"
    assert detect_format("<arg_key>") == "glm45"


def test_chat_service_uses_template_format():
    from octopus_b200.serving.chat import ChatTokenizer
    from octopus_b200.serving.local import ChatService
    from test_engine_cpu import tiny_engine

    _, _, eng = tiny_engine()
    svc = ChatService(eng, ChatTokenizer.tiny())
    assert svc.tool_format == "qwen25"
    assert ChatService(eng, ChatTokenizer.tiny(), tool_format="qwen3_coder").tool_format == "qwen3_coder"
