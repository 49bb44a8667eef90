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


def test_measure_sweep_over_two_gpus_equals_one(tmp_path):
    """The config-4 sweep split by piece over two GPUs (torch.distributed.run, NCCL, records gathered on every rank)
    gives the one-GPU sweep's records, KL for KL."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import json
    from lookatmyquant_b200 import measure
    out = tmp_path / "two.json"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
                        "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", "29561", "-m",
                        "lookatmyquant_b200.measure", "--layers", "0:2", "--model-layers", "2", "--windows", "2",
                        "--T", "128", "--calib", "2", "--options", "tr2", "--out", str(out)],
                       capture_output=True, text=True, env=env)
    print(r.stdout[-4000:], r.stderr[-4000:])
    assert r.returncode == 0
    two = json.loads(out.read_text())
    one = measure.run(layers=range(2), options=("tr2",), n_layers=2, windows=2, T=128, calib=2, log=lambda s: None)
    assert two["world"] == 2 and two["probes"] == one["probes"] == 14
    assert [(x["item"], x["option"], x["dkl"]) for x in two["records"]] == \
        [(x["item"], x["option"], x["dkl"]) for x in one["records"]]
