"""Fold a PEFT LoRA adapter into an HF safetensors checkpoint (W + alpha/r B A), so the
merged directory serves like the base (same config, tokenizer and other files).

    python -m octopus_b200.tools.tree_sft.merge_lora --adapter RUN/final --base HF_DIR --out DIR

Adapter keys `base_model.model.model.layers.<i>.<parent>.<module>.lora_{A,B}.weight` map to
the checkpoint's `model.layers.<i>.<parent>.<module>.weight` (or the same under
`model.language_model.` for multimodal wrappers); a target missing from the checkpoint is an
error.  The merge runs in fp32 and is stored in each weight's own dtype.

Reference parity (behaviour): `octopus/tools/tree_sft/merge_lora.py:1-63`.
"""
from __future__ import annotations

import argparse
import json
import re
import shutil
from pathlib import Path

import torch

_KEY = re.compile(r"base_model\.model\.model\.(layers\.\d+\..+)\.lora_([AB])(?:\.default)?\.weight$")


def lora_deltas(adapter) -> dict[str, torch.Tensor]:
    """{"layers.<i>.<parent>.<module>": s * B @ A} in fp32."""
    from safetensors.torch import load_file

    adapter = Path(adapter)
    cfg = json.loads((adapter / "adapter_config.json").read_text())
    scale = float(cfg["lora_alpha"]) / float(cfg["r"])
    pairs: dict[str, dict] = {}
    for key, t in load_file(str(adapter / "adapter_model.safetensors")).items():
        m = _KEY.match(key)
        if not m:
            raise ValueError(f"unexpected adapter key {key}")
        pairs.setdefault(m.group(1), {})[m.group(2)] = t.float()
    return {name: (ab["B"] @ ab["A"]) * scale for name, ab in pairs.items()}


def _weight_map(base: Path) -> dict:
    idx = base / "model.safetensors.index.json"
    if idx.is_file():
        return json.loads(idx.read_text())["weight_map"]
    from safetensors import safe_open

    out = {}
    for f in sorted(base.glob("*.safetensors")):
        with safe_open(str(f), framework="pt") as h:
            out.update({k: f.name for k in h.keys()})
    return out


def merge(adapter, base, out) -> int:
    from safetensors.torch import load_file, save_file

    base, out = Path(base), Path(out)
    deltas = lora_deltas(adapter)
    wmap = _weight_map(base)
    names = {}
    for mod in deltas:
        for pre in ("model.", "model.language_model."):
            if f"{pre}{mod}.weight" in wmap:
                names[f"{pre}{mod}.weight"] = mod
                break
        else:
            raise KeyError(f"LoRA target {mod} is not in the checkpoint at {base}")
    out.mkdir(parents=True, exist_ok=True)
    merged = 0
    for shard in sorted(set(wmap.values())):
        tensors = load_file(str(base / shard))
        for name in [n for n in tensors if n in names]:
            tensors[name] = (tensors[name].float() + deltas[names[name]]).to(tensors[name].dtype)
            merged += 1
        save_file(tensors, str(out / shard), metadata={"format": "pt"})
    for f in base.iterdir():
        if f.is_file() and not f.name.endswith(".safetensors"):
            shutil.copy2(f, out / f.name)
    (out / "MERGED_FROM.json").write_text(json.dumps({"base": str(base), "adapter": str(Path(adapter).resolve()),
                                                      "weights_merged": merged}, indent=1))
    return merged


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m octopus_b200.tools.tree_sft.merge_lora")
    ap.add_argument("--adapter", required=True)
    ap.add_argument("--base", required=True)
    ap.add_argument("--out", required=True)
    args = ap.parse_args(argv)
    print(f"merged {merge(args.adapter, args.base, args.out)} weights from {args.adapter} into {args.out}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
