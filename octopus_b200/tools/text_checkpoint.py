"""Vision-language checkpoint -> text-only HF safetensors checkpoint.

    python -m octopus_b200.tools.text_checkpoint SRC_DIR DST_DIR

Keeps the language model's tensors (`model.language_model.X` -> `model.X`, and
`lm_head.weight`), drops the vision tower and projector, and writes the shards, the
weight index and a text config (the source's `text_config` when present).

Reference parity (behaviour): `octopus/rl/text_checkpoint.py:1-56`.
"""
from __future__ import annotations

import glob
import json
import os
import sys

LM_PREFIXES = (("model.language_model.", "model."), ("language_model.model.", "model."),
               ("language_model.lm_head.", "lm_head."), ("lm_head.", "lm_head."), ("model.", "model."))
DROP = ("model.visual.", "visual.", "model.vision_tower.", "vision_tower.", "model.multi_modal_projector.",
        "multi_modal_projector.", "model.vision_model.")


def text_name(key: str) -> str | None:
    if key.startswith(DROP):
        return None
    for src, dst in LM_PREFIXES:
        if key.startswith(src):
            return dst + key[len(src):]
    return None


def convert(src: str, dst: str, max_shard_bytes: int = 5 << 30) -> dict:
    from safetensors import safe_open
    from safetensors.torch import save_file

    os.makedirs(dst, exist_ok=True)
    tensors = {}
    for fn in sorted(glob.glob(os.path.join(src, "*.safetensors"))):
        with safe_open(fn, framework="pt") as f:
            for k in f.keys():
                n = text_name(k)
                if n is not None:
                    tensors[n] = f.get_tensor(k)
    if not tensors:
        raise ValueError(f"no language-model tensors under {src}")
    shards, cur, size = [], {}, 0
    for k in sorted(tensors):
        nb = tensors[k].numel() * tensors[k].element_size()
        if cur and size + nb > max_shard_bytes:
            shards.append(cur)
            cur, size = {}, 0
        cur[k] = tensors[k]
        size += nb
    shards.append(cur)
    index = {"metadata": {"total_size": sum(t.numel() * t.element_size() for t in tensors.values())},
             "weight_map": {}}
    for i, sh in enumerate(shards):
        name = f"model-{i + 1:05d}-of-{len(shards):05d}.safetensors"
        save_file({k: v.contiguous() for k, v in sh.items()}, os.path.join(dst, name))
        for k in sh:
            index["weight_map"][k] = name
    with open(os.path.join(dst, "model.safetensors.index.json"), "w") as f:
        json.dump(index, f, indent=1)
    cfg_path = os.path.join(src, "config.json")
    if os.path.exists(cfg_path):
        cfg = json.load(open(cfg_path))
        text = dict(cfg.get("text_config") or cfg)
        text.pop("vision_config", None)
        text.setdefault("architectures", ["Qwen2ForCausalLM"])
        with open(os.path.join(dst, "config.json"), "w") as f:
            json.dump(text, f, indent=1)
    for aux in ("tokenizer.json", "tokenizer_config.json", "chat_template.jinja", "generation_config.json"):
        p = os.path.join(src, aux)
        if os.path.exists(p):
            with open(p, "rb") as a, open(os.path.join(dst, aux), "wb") as b:
                b.write(a.read())
    return {"tensors": len(tensors), "shards": len(shards)}


def main(argv=None) -> int:
    argv = sys.argv[1:] if argv is None else argv
    if len(argv) != 2:
        print(__doc__)
        return 2
    print(json.dumps(convert(argv[0], argv[1])))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
