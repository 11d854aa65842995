"""Tool-call parsers of model outputs, one per chat-template family: a completion's text ->
(content, OpenAI tool_calls).  The serving side of the runtime's tool-call formats
(runtime/core.py TOOL_FORMATS: which markup a model emits); `detect_format` picks the family
from a chat template.

  qwen25 / hermes   <tool_call>{"name": ..., "arguments": {...}}</tool_call>
  qwen3_coder       <tool_call><function=NAME><parameter=KEY>VALUE</parameter>...</function></tool_call>
                    (values are text; a parameter the tool's schema types as non-string is
                    read as JSON when it parses)
  llama3            [<|python_tag|>]{"name": ..., "parameters": {...}} (several joined by ';')
  mistral           [TOOL_CALLS][{"name": ..., "arguments": {...}}, ...] or
                    [TOOL_CALLS]NAME[ARGS]{...} (repeated)
  deepseekv3        <｜tool▁call▁begin｜>function<｜tool▁sep｜>NAME\n```json\n{...}\n```<｜tool▁call▁end｜>
  deepseekv31       <｜tool▁call▁begin｜>NAME<｜tool▁sep｜>{...}<｜tool▁call▁end｜>
  glm45             <tool_call>NAME\n<arg_key>K</arg_key>\n<arg_value>V</arg_value>...</tool_call>
  kimi_k2           <|tool_call_begin|>functions.NAME:IDX<|tool_call_argument_begin|>{...}<|tool_call_end|>
  gpt-oss           ...to=functions.NAME ...<|message|>{...}<|call|>
Malformed calls are left in the content (no call is invented).

Reference parity (behaviour): the SGLang tool-call parser families named by the runtime's
formats (`octopus/runtime/core.py:33-56`); the reference serves through SGLang's detectors.
"""
from __future__ import annotations

import json
import re
import uuid

_ALIASES = {"hermes": "qwen25", "qwen": "qwen25", "step3p5": "qwen3_coder", "glm": "glm45", "glm47": "glm45"}


def _call(name: str, args) -> dict:
    return {"id": f"call_{uuid.uuid4().hex[:9]}", "type": "function",
            "function": {"name": name, "arguments": args if isinstance(args, str) else json.dumps(args)}}


def _json_obj(text: str):
    try:
        v = json.loads(text)
    except (json.JSONDecodeError, TypeError):
        return None
    return v if isinstance(v, dict) else None


def _schema_types(tools, name: str) -> dict:
    for t in tools or []:
        fn = t.get("function") or t
        if fn.get("name") == name:
            return {k: (v or {}).get("type") for k, v in ((fn.get("parameters") or {}).get("properties") or {}).items()}
    return {}


def _typed(value: str, typ) -> object:
    """A text parameter value as its schema type (JSON when it parses; text otherwise)."""
    if typ in (None, "string"):
        return value
    try:
        return json.loads(value)
    except json.JSONDecodeError:
        return value


def _strip(text: str, spans) -> str:
    out, last = [], 0
    for a, b in spans:
        out.append(text[last:a])
        last = b
    out.append(text[last:])
    return "".join(out).strip()


def _qwen25(text, tools):
    calls, spans = [], []
    for m in re.finditer(r"<tool_call>\s*(\{.*?\})\s*</tool_call>", text, re.S):
        obj = _json_obj(m.group(1))
        if obj is None or not isinstance(obj.get("name"), str):
            continue
        calls.append(_call(obj["name"], obj.get("arguments", {})))
        spans.append(m.span())
    return calls, spans


def _qwen3_coder(text, tools):
    calls, spans = [], []
    for m in re.finditer(r"(?:<tool_call>\s*)?<function=([^>\n]+)>(.*?)</function>(?:\s*</tool_call>)?", text, re.S):
        name = m.group(1).strip()
        types = _schema_types(tools, name)
        args = {}
        for p in re.finditer(r"<parameter=([^>\n]+)>(.*?)</parameter>", m.group(2), re.S):
            key = p.group(1).strip()
            val = p.group(2)
            val = val[1:] if val.startswith("\n") else val
            val = val[:-1] if val.endswith("\n") else val
            args[key] = _typed(val, types.get(key))
        calls.append(_call(name, args))
        spans.append(m.span())
    return calls, spans


def _llama3(text, tools):
    body = text.split("<|python_tag|>", 1)[1] if "<|python_tag|>" in text else text.strip()
    start = text.find(body) if body else -1
    calls = []
    for part in body.split(";"):
        obj = _json_obj(part.strip())
        if obj is None or not isinstance(obj.get("name"), str):
            return [], []
        calls.append(_call(obj["name"], obj.get("parameters", obj.get("arguments", {}))))
    if not calls:
        return [], []
    a = text.find("<|python_tag|>")
    return calls, [((a if a >= 0 else start), len(text))]


def _mistral(text, tools):
    i = text.find("[TOOL_CALLS]")
    if i < 0:
        return [], []
    rest = text[i + len("[TOOL_CALLS]"):].lstrip()
    dec = json.JSONDecoder()
    if rest.startswith("["):
        try:
            arr, _ = dec.raw_decode(rest)
        except json.JSONDecodeError:
            return [], []
        calls = [_call(o["name"], o.get("arguments", {})) for o in arr if isinstance(o, dict) and "name" in o]
        return calls, [(i, len(text))] if calls else []
    calls, pos, body = [], 0, text[i:].replace("[TOOL_CALLS]", " ")
    head = re.compile(r"\s*([^\[\s]+)(?:\[CALL_ID\][^\[]*)?\[ARGS\]")
    while True:
        m = head.match(body, pos)
        if not m:
            break
        try:
            obj, end = dec.raw_decode(body, m.end())
        except json.JSONDecodeError:
            break
        if isinstance(obj, dict):
            calls.append(_call(m.group(1), obj))
        pos = end
    return calls, [(i, len(text))] if calls else []


def _deepseekv3(text, tools):
    calls, spans = [], []
    pat = r"<｜tool▁call▁begin｜>function<｜tool▁sep｜>([^\n]+)\n```json\n(.*?)\n```<｜tool▁call▁end｜>"
    for m in re.finditer(pat, text, re.S):
        obj = _json_obj(m.group(2))
        if obj is not None:
            calls.append(_call(m.group(1).strip(), obj))
            spans.append(m.span())
    return calls, _outer(text, spans, "<｜tool▁calls▁begin｜>", "<｜tool▁calls▁end｜>")


def _deepseekv31(text, tools):
    calls, spans = [], []
    for m in re.finditer(r"<｜tool▁call▁begin｜>([^<]+)<｜tool▁sep｜>(.*?)<｜tool▁call▁end｜>", text, re.S):
        obj = _json_obj(m.group(2))
        if obj is not None:
            calls.append(_call(m.group(1).strip(), obj))
            spans.append(m.span())
    return calls, _outer(text, spans, "<｜tool▁calls▁begin｜>", "<｜tool▁calls▁end｜>")


def _outer(text, spans, begin, end):
    """Widen call spans to the enclosing calls block when present."""
    if not spans:
        return spans
    a, b = text.find(begin), text.rfind(end)
    if a >= 0 and b >= 0:
        return [(a, b + len(end))]
    return spans


def _glm45(text, tools):
    calls, spans = [], []
    for m in re.finditer(r"<tool_call>([^\n<]+)(.*?)</tool_call>", text, re.S):
        name = m.group(1).strip()
        types = _schema_types(tools, name)
        args = {}
        for p in re.finditer(r"<arg_key>(.*?)</arg_key>\s*<arg_value>(.*?)</arg_value>", m.group(2), re.S):
            args[p.group(1).strip()] = _typed(p.group(2), types.get(p.group(1).strip()))
        calls.append(_call(name, args))
        spans.append(m.span())
    return calls, spans


def _kimi_k2(text, tools):
    calls, spans = [], []
    pat = (r"<\|tool_call_begin\|>\s*(?:functions\.)?([\w.\-]+):\d+\s*<\|tool_call_argument_begin\|>(.*?)"
           r"<\|tool_call_end\|>")
    for m in re.finditer(pat, text, re.S):
        obj = _json_obj(m.group(2).strip())
        if obj is not None:
            calls.append(_call(m.group(1), obj))
            spans.append(m.span())
    return calls, _outer(text, spans, "<|tool_calls_section_begin|>", "<|tool_calls_section_end|>")


def _gpt_oss(text, tools):
    calls, spans = [], []
    for m in re.finditer(r"to=functions\.([^\s<]+).*?<\|message\|>(.*?)<\|call\|>", text, re.S):
        obj = _json_obj(m.group(2).strip())
        if obj is not None:
            calls.append(_call(m.group(1), obj))
            spans.append(m.span())
    return calls, spans


PARSERS = {"qwen25": _qwen25, "qwen3_coder": _qwen3_coder, "llama3": _llama3, "mistral": _mistral,
           "deepseekv3": _deepseekv3, "deepseekv31": _deepseekv31, "glm45": _glm45, "kimi_k2": _kimi_k2,
           "gpt-oss": _gpt_oss}


def parse(text: str, fmt: str = "qwen25", tools=None) -> tuple[str, list[dict]]:
    """(content, tool_calls) of a completion in format `fmt` (the text unchanged when it has
    no well-formed call)."""
    fmt = _ALIASES.get(fmt, fmt)
    if fmt not in PARSERS:
        raise ValueError(f"tool-call format {fmt!r} is none of {sorted(PARSERS)}")
    calls, spans = PARSERS[fmt](text, tools)
    if not calls:
        return text, []
    return _strip(text, spans), calls


def detect_format(template: str | None) -> str:
    """The tool-call family a chat template renders (qwen25 when nothing more specific shows)."""
    t = template or ""
    for marker, fmt in (("<function=", "qwen3_coder"), ("<arg_key>", "glm45"),
                        ("function<｜tool▁sep｜>", "deepseekv3"), ("tool▁call▁begin", "deepseekv31"),
                        ("<|tool_call_begin|>", "kimi_k2"), ("to=functions", "gpt-oss"), ("[TOOL_CALLS]", "mistral"),
                        ("<|python_tag|>", "llama3"), ("<tool_call>", "qwen25")):
        if marker in t:
            return fmt
    return "qwen25"


__all__ = ["PARSERS", "detect_format", "parse"]
