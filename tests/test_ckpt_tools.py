"""Text-only checkpoint conversion and the adapter push (fake ssh) on CPU."""
import json
import os
import stat

import pytest
import torch
from safetensors.torch import load_file, save_file

from octopus_b200.rl.adapter_push import PushError, push_adapter
from octopus_b200.tools.text_checkpoint import convert


def test_text_checkpoint(tmp_path):
    src = tmp_path / "vl"
    src.mkdir()
    save_file({"model.language_model.layers.0.mlp.up_proj.weight": torch.ones(4, 2),
               "model.language_model.embed_tokens.weight": torch.zeros(8, 2),
               "lm_head.weight": torch.ones(8, 2), "model.visual.blocks.0.w": torch.ones(3)},
              str(src / "model-00001-of-00001.safetensors"))
    json.dump({"model_type": "qwen2_5_vl", "text_config": {"hidden_size": 2}, "vision_config": {}},
              open(src / "config.json", "w"))
    out = convert(str(src), str(tmp_path / "txt"))
    assert out["tensors"] == 3
    d = load_file(str(tmp_path / "txt" / "model-00001-of-00001.safetensors"))
    assert set(d) == {"model.layers.0.mlp.up_proj.weight", "model.embed_tokens.weight", "lm_head.weight"}
    assert json.load(open(tmp_path / "txt" / "config.json"))["hidden_size"] == 2


def _fake_ssh(tmp_path, fail_first: int):
    """An ssh stand-in: exits 255 the first `fail_first` times, then runs the command locally."""
    cnt = tmp_path / "count"
    cnt.write_text("0")
    p = tmp_path / "fakessh"
    p.write_text(f"""#!/bin/bash
n=$(cat {cnt}); echo $((n+1)) > {cnt}
if [ "$n" -lt {fail_first} ]; then cat > /dev/null; exit 255; fi
shift; bash -c "$1"
""")
    p.chmod(p.stat().st_mode | stat.S_IEXEC)
    return str(p)


def test_adapter_push_retries(tmp_path):
    src = tmp_path / "ad"
    src.mkdir()
    (src / "adapter_model.safetensors").write_bytes(b"abc")
    dest = tmp_path / "remote" / "v3"
    ssh = _fake_ssh(tmp_path, fail_first=1)
    res = push_adapter(str(src), ["hostA"], str(dest), ssh=(ssh,), sleep=lambda s: None)
    assert res == {"hostA": 2}
    assert (dest / "adapter_model.safetensors").read_bytes() == b"abc"
    ssh2 = _fake_ssh(tmp_path, fail_first=5)
    with pytest.raises(PushError):
        push_adapter(str(src), ["hostB"], str(dest), ssh=(ssh2,), retries=2, sleep=lambda s: None)
