import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
GOLDEN = ROOT / "tests" / "golden"
TABLES = ROOT / "lookatmyquant_b200" / "tables"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (a B200) and the built liblamq_b200.so")


def table(k):
    return np.fromfile(TABLES / f"trellis_L12_k{k}_T256_s0_ema.f64", dtype="<f8")


@pytest.fixture(scope="session")
def golden():
    cache = {}

    def load(name):
        if name not in cache:
            cache[name] = dict(np.load(GOLDEN / f"{name}.npz"))
        return cache[name]
    return load
