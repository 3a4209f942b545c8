"""Sharded stack on two GPUs: peer-store exchange and NCCL all-gather against the unsharded stack.

Needs at least two GPUs of one node (skipped otherwise); the ranks run as separate processes under
torchrun, one per GPU, and each is bounded by a timeout.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

WORKER = Path(__file__).resolve().parent / "multi_gpu_worker.py"


@pytest.mark.gpu
def test_sharded_stack_two_gpus_bit_identical():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29533", str(WORKER)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    out = r.stdout + r.stderr
    assert r.returncode == 0, out[-4000:]
    assert out.count(": ok") == 2, out[-4000:]
