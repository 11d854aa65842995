"""Tensor-parallel fused kernels and the TP rollout engine on 2 GPUs (one rank per GPU,
launched by torchrun; the per-rank checks are in tests/_tp_worker.py)."""
import os
import socket
import subprocess
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.gpu
def test_tp_fused_kernels_and_engine():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs (one rank per GPU)")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=ROOT)
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(ROOT, "tests", "_tp_worker.py")]
    p = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True)
    out = p.stdout + p.stderr
    print(out[-4000:])
    assert p.returncode == 0, out[-4000:]
    for name in ("ag rows_s=8", "ag rows_s=512", "rs rows_s=256", "rs-norm rows_s=16", "sample", "engine forward",
                 "engine generate", "engine reshard", "fsdp fused master", "fsdp fused weights",
                 "fsdp full-shard master", "fsdp full-shard weights"):
        assert f"TP_OK {name}" in out, name
