"""The layer build over two and four GPUs (one process per GPU, NCCL) against the one-GPU build. Each case runs only
where the box has that many GPUs."""

import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("ranks", [2, 4])
def test_multi_gpu_layer_matches_one_gpu(ranks):
    if not torch.cuda.is_available() or torch.cuda.device_count() < ranks:
        pytest.skip(f"needs {ranks} GPUs")
    here = Path(__file__).resolve().parent
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
                        "--nproc-per-node", str(ranks), "--master-addr", "127.0.0.1", "--master-port",
                        str(29533 + ranks), str(here / "dist_layer_check.py")], capture_output=True, text=True, env=env)
    print(r.stdout[-4000:], r.stderr[-4000:])
    assert r.returncode == 0
