"""Chat layer: tokenizer + chat template, tool-call parsing, and the cursor delta renderer.

`render_delta` returns the prompt token ids that extend a cursor by new messages, at a
cost independent of the history: the new messages are rendered after a constant stub
conversation that ends on an assistant reply (as every cursor does), and only the text
after the stub reply's terminator is tokenized.  The template's turn markers are
special tokens, so tokenization never merges across that boundary and the ids equal
the tail of tokenizing the whole conversation (`concat_oracle`).  `terminator` gives
the tokens a template renders after a reply in place of the model's stop token; a
cursor's tokens are prompt + reply without stop + terminator.

`ChatTokenizer` loads an HF tokenizer directory (tokenizer.json + tokenizer_config.json
chat template) through the `tokenizers` library and a sandboxed jinja2 renderer, or is
built in-process (`ChatTokenizer.tiny`) with a ChatML template for tests.

Reference parity: `octopus/serving/delta_render.py:29-281` (render_delta, terminator,
stub probing, concat oracle), `octopus/serving/cursor_store.py:put_reply` (stop stripped,
terminator appended).
"""
from __future__ import annotations

import json
import os

STUB = [{"role": "user", "content": "stub"}, {"role": "assistant", "content": "stub"}]

CHATML_TEMPLATE = (
    "{% if tools %}<|im_start|>system\n{% if messages[0]['role'] == 'system' %}{{ messages[0]['content'] }}\n\n"
    "{% endif %}# Tools\n<tools>{% for t in tools %}\n{{ t | tojson }}{% endfor %}\n</tools>\nCall a tool as "
    "<tool_call>{\"name\": ..., \"arguments\": ...}</tool_call><|im_end|>\n"
    "{% elif messages[0]['role'] == 'system' %}<|im_start|>system\n{{ messages[0]['content'] }}<|im_end|>\n{% endif %}"
    "{% for m in messages %}"
    "{% if m['role'] == 'system' and loop.first %}"
    "{% elif m['role'] == 'assistant' %}<|im_start|>assistant\n{{ m['content'] or '' }}"
    "{% for c in (m['tool_calls'] or []) %}\n<tool_call>\n{\"name\": \"{{ c['function']['name'] }}\", "
    "\"arguments\": {{ c['function']['arguments'] if c['function']['arguments'] is string else "
    "(c['function']['arguments'] | tojson) }}}\n</tool_call>{% endfor %}<|im_end|>\n"
    "{% elif m['role'] == 'tool' %}<|im_start|>user\n<tool_response>\n{{ m['content'] }}\n</tool_response><|im_end|>\n"
    "{% else %}<|im_start|>{{ m['role'] }}\n{{ m['content'] }}<|im_end|>\n{% endif %}"
    "{% endfor %}"
    "{% if add_generation_prompt %}<|im_start|>assistant\n{% endif %}"
)


def _env():
    import jinja2.ext
    import jinja2.sandbox

    def raise_exception(msg):
        raise jinja2.TemplateError(msg)

    env = jinja2.sandbox.ImmutableSandboxedEnvironment(trim_blocks=True, lstrip_blocks=True,
                                                       extensions=[jinja2.ext.loopcontrols])
    env.filters["tojson"] = lambda x, ensure_ascii=False, indent=None, separators=None, sort_keys=False: json.dumps(
        x, ensure_ascii=ensure_ascii, indent=indent, separators=separators, sort_keys=sort_keys)
    env.globals["raise_exception"] = raise_exception
    return env


class ChatTokenizer:
    def __init__(self, tokenizer, template: str, eos: str = "<|im_end|>", stop_ids=None):
        self.tok = tokenizer
        self.template_src = template
        self.template = _env().from_string(template)
        self.eos = eos
        self.eos_id = tokenizer.token_to_id(eos)
        self.stop_ids = tuple(stop_ids) if stop_ids else ((self.eos_id,) if self.eos_id is not None else ())
        self._term = None

    # ------------------------------------------------------------------ construction
    @staticmethod
    def from_dir(path: str) -> "ChatTokenizer":
        from tokenizers import Tokenizer

        tok = Tokenizer.from_file(os.path.join(path, "tokenizer.json"))
        tmpl = None
        tp = os.path.join(path, "chat_template.jinja")
        if os.path.exists(tp):
            tmpl = open(tp).read()
        cfg = {}
        cp = os.path.join(path, "tokenizer_config.json")
        if os.path.exists(cp):
            cfg = json.load(open(cp))
            tmpl = tmpl or cfg.get("chat_template")
        eos = cfg.get("eos_token") or "<|im_end|>"
        if isinstance(eos, dict):
            eos = eos.get("content")
        return ChatTokenizer(tok, tmpl or CHATML_TEMPLATE, eos)

    @staticmethod
    def tiny(vocab_words: int = 2000) -> "ChatTokenizer":
        """A small word-level tokenizer with ChatML specials (tests, synthetic runs)."""
        from tokenizers import Tokenizer, models, pre_tokenizers, decoders

        specials = ["<|endoftext|>", "<|im_start|>", "<|im_end|>", "<unk>"]
        base = list("abcdefghijklmnopqrstuvwxyzABCDEFGHIJKLMNOPQRSTUVWXYZ0123456789") + \
            list(".,:;!?-_/\\'\"()[]{}<>=+*#@$%&|~`^ \n\t")
        vocab = {t: i for i, t in enumerate(specials + base)}
        tok = Tokenizer(models.WordPiece(vocab, unk_token="<unk>", max_input_chars_per_word=10_000))
        tok.add_special_tokens(specials)
        tok.pre_tokenizer = pre_tokenizers.Split("", behavior="isolated")
        tok.decoder = decoders.Fuse()
        return ChatTokenizer(tok, CHATML_TEMPLATE, "<|im_end|>")

    # ------------------------------------------------------------------ basics
    @property
    def vocab_size(self) -> int:
        return self.tok.get_vocab_size()

    def encode(self, text: str) -> list[int]:
        return self.tok.encode(text, add_special_tokens=False).ids

    def decode(self, ids) -> str:
        return self.tok.decode([int(i) for i in ids], skip_special_tokens=False)

    def render(self, messages: list[dict], tools: list | None = None, add_generation_prompt: bool = False,
               **kwargs) -> str:
        return self.template.render(messages=messages, tools=tools, add_generation_prompt=add_generation_prompt,
                                    **kwargs)

    def apply(self, messages, tools=None, add_generation_prompt=True, **kwargs) -> list[int]:
        return self.encode(self.render(messages, tools, add_generation_prompt, **kwargs))

    # ------------------------------------------------------------------ cursor protocol
    def terminator(self) -> list[int]:
        """Tokens the template renders after an assistant reply (in place of its stop token)."""
        if self._term is None:
            text = self.render(STUB)
            i = text.rindex("stub") + len("stub")
            self._term = self.encode(text[i:])
        return list(self._term)

    def render_delta(self, messages: list[dict], tools: list | None = None, **kwargs) -> list[int]:
        """Prompt ids extending a cursor by `messages` (with the generation prompt)."""
        stub = self.render(STUB, tools, False, **kwargs)
        full = self.render(STUB + list(messages), tools, True, **kwargs)
        if not full.startswith(stub):
            raise ValueError("chat template renders the history differently after new messages; delta rendering "
                             "needs a history-independent template")
        return self.encode(full[len(stub):])

    def concat_oracle(self, history: list[dict], messages: list[dict], tools=None, **kwargs) -> list[int]:
        """The tail of tokenizing the whole conversation after the history's last reply terminator."""
        head = self.encode(self.render(history, tools, False, **kwargs))
        full = self.encode(self.render(history + list(messages), tools, True, **kwargs))
        assert full[:len(head)] == head, "whole-conversation tokens do not extend the history's"
        return full[len(head):]

    def reply_tokens(self, output_ids: list[int]) -> list[int]:
        """A reply as a cursor keeps it: output without trailing stop tokens + terminator."""
        out = list(output_ids)
        while out and out[-1] in self.stop_ids:
            out.pop()
        return out + self.terminator()


def parse_tool_calls(text: str, fmt: str = "qwen25", tools=None) -> tuple[str, list[dict]]:
    """Split a completion into (content, OpenAI tool_calls) for tool-call format `fmt`
    (serving.tool_parsers; hermes / qwen25 by default)."""
    from .tool_parsers import parse

    return parse(text, fmt, tools)
