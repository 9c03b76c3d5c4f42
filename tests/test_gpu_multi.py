"""The N-split on several GPUs of one node: the fused GEMM + all-gather over NVLink.

Runs tests/multi_gpu_worker.py under torch.distributed.run with one rank per visible
GPU (up to 8); every rank checks the fused and the NCCL-gathered outputs against its
own 1-GPU result bit for bit. Skipped with fewer than two GPUs.
"""

from __future__ import annotations

import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

WORKER = Path(__file__).resolve().parent / "multi_gpu_worker.py"


def free_port() -> int:
    with socket.socket() as probe:
        probe.bind(("127.0.0.1", 0))
        return int(probe.getsockname()[1])


def test_fused_gemm_all_gather_matches_one_gpu() -> None:
    import torch

    gpus = torch.cuda.device_count()
    if gpus < 2:
        pytest.skip("needs at least two GPUs")
    world = min(gpus, 8)
    command = [
        "timeout", "-k", "30", "600",
        sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}",
        "--master-addr", "127.0.0.1", f"--master-port={free_port()}", str(WORKER),
    ]
    result = subprocess.run(command, capture_output=True, text=True, timeout=700, env=dict(os.environ))
    assert result.returncode == 0, (result.stdout[-4000:], result.stderr[-4000:])
    assert result.stdout.count(": ok") == world
