"""The C-ABI library builds, loads and exports every entry point include/lamq_b200.h declares (no GPU needed)."""

import ctypes
import re
from pathlib import Path

import pytest

from lookatmyquant_b200 import _lib
from lookatmyquant_b200.build import LIB, build

HEADER = Path(__file__).resolve().parents[1] / "include" / "lamq_b200.h"


def declared():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(lamq_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    if not LIB.exists():
        build()
    return _lib.load()


def test_every_declared_symbol_is_exported(lib):
    names = declared()
    assert "lamq_viterbi" in names and "lamq_ldlq_rowtrellis" in names
    for name in names:
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_abi_version_and_errors_without_gpu(lib):
    assert lib.lamq_abi_version() >= 1
    # argument validation happens before any CUDA call
    st = lib.lamq_viterbi(None, 4, 8, None, 11, 2, None, None, None, 0, None)
    assert st == _lib.LAMQ_ERR_INVALID
    assert b"L = 12" in lib.lamq_last_error()
    st = lib.lamq_ldlq_rowtrellis(None, 16, 4, 16, None, 16, None, None, None, None, 2, 12, 16, 20, 128,
                                  None, None, None, 0, None)
    assert st == _lib.LAMQ_ERR_INVALID
    assert lib.lamq_viterbi(None, 0, 8, None, 12, 2, None, None, None, 0, None) == _lib.LAMQ_OK  # empty input


def test_workspace_sizes(lib):
    assert lib.lamq_viterbi_workspace_size(100, 24, 12, 2) == 0  # short sequences keep back-pointers on chip
    assert lib.lamq_viterbi_workspace_size(3, 256, 12, 2) == 3 * 256 * 32 * 8
