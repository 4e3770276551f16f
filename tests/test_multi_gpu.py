"""Block-row-sharded S+LR layers over NCCL equal the single-GPU forward.

Needs at least two GPUs; launches tests/multi_gpu_check.py under torchrun
(one process per GPU, rendezvous on 127.0.0.1)."""
from __future__ import annotations

import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
HERE = Path(__file__).resolve().parent


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two or more GPUs")
def test_sharded_forward_equals_single_gpu():
    n = min(torch.cuda.device_count(), 8)
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr=127.0.0.1", f"--master-port={_port()}",
           str(HERE / "multi_gpu_check.py")]
    res = subprocess.run(cmd, capture_output=True, text=True, env={**__import__("os").environ, "NCCL_NVLS_ENABLE": "0"})
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
    assert "MISMATCH" not in res.stdout
