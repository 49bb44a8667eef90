"""The layer build over two GPUs (one process per GPU, NCCL) against the one-GPU build. Runs only where the box has
two or more GPUs."""

import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_layer_matches_one_gpu():
    here = Path(__file__).resolve().parent
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
                        "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", "29533",
                        str(here / "dist_layer_check.py")], capture_output=True, text=True, env=env)
    print(r.stdout[-4000:], r.stderr[-4000:])
    assert r.returncode == 0
