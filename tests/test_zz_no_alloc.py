"""The allocation-free Viterbi entry point (lamq_viterbi_noalloc) against lamq_viterbi, through the C ABI.

lamq_viterbi_noalloc exists for callers that cannot allocate device memory (a host whose own pool owns the device,
an FFI binding without a device allocator): it keeps long sequences' back-pointers in a scratch array built into the
library instead of a caller-provided workspace. Its states must equal lamq_viterbi's exactly (the tolerance of every
Viterbi test here: bit-exact), on two calls in a row — the second call reuses the array the first one left behind.
This file is collected last so a failure here cannot hide the other tests' results.
"""

import numpy as np
import pytest
import torch

from conftest import GOLDEN, table
from lookatmyquant_b200 import _lib


def _viterbi_ws(lib, X, V, start, k):
    rows, T = X.shape
    out = torch.empty(rows, T, dtype=torch.int64, device="cuda")
    ws = lib.lamq_viterbi_workspace_size(rows, T, 12, k)
    buf = torch.empty(max(ws, 1), dtype=torch.uint8, device="cuda")
    _lib.check(lib.lamq_viterbi(X.data_ptr(), rows, T, V.data_ptr(), 12, k,
                                None if start is None else start.data_ptr(), out.data_ptr(), buf.data_ptr(), ws,
                                torch.cuda.current_stream().cuda_stream), "lamq_viterbi")
    return out


def _viterbi_noalloc(lib, X, V, start, k):
    rows, T = X.shape
    out = torch.empty(rows, T, dtype=torch.int64, device="cuda")
    _lib.check(lib.lamq_viterbi_noalloc(X.data_ptr(), rows, T, V.data_ptr(), 12, k,
                                        None if start is None else start.data_ptr(), out.data_ptr(),
                                        torch.cuda.current_stream().cuda_stream), "lamq_viterbi_noalloc")
    return out


def test_noalloc_rejects_oversized_input_without_a_gpu():
    lib = _lib.load()
    # 1024 sequences of 256 entries need 64 MiB of back-pointers, more than the built-in 32 MiB
    assert lib.lamq_viterbi_noalloc(None, 1024, 256, None, 12, 2, None, None, None) == _lib.LAMQ_ERR_INVALID
    assert b"use lamq_viterbi with a workspace" in lib.lamq_last_error()


@pytest.mark.gpu
@pytest.mark.parametrize("k", [1, 2, 3, 4])
def test_noalloc_matches_workspace_entry_point_twice(k):
    lib = _lib.load()
    V = torch.as_tensor(table(k)).float().cuda()
    rng = np.random.default_rng(7 + k)
    for call, (rows, T, with_start) in enumerate([(512, 256, False), (300, 200, True)]):  # two calls in a row
        X = torch.as_tensor(rng.standard_normal((rows, T)), dtype=torch.float32).cuda()
        start = torch.as_tensor(rng.integers(0, 4096, rows)).cuda() if with_start else None
        got = _viterbi_noalloc(lib, X, V, start, k)
        want = _viterbi_ws(lib, X, V, start, k)
        torch.cuda.synchronize()
        assert torch.equal(got, want), f"call {call}: states differ"
    # short windows need no scratch at all
    X = torch.as_tensor(rng.standard_normal((1000, 24)), dtype=torch.float32).cuda()
    start = torch.as_tensor(rng.integers(0, 4096, 1000)).cuda()
    assert torch.equal(_viterbi_noalloc(lib, X, V, start, k), _viterbi_ws(lib, X, V, start, k))
    # and the reference's own paths (tests/golden/viterbi.npz: free-start sequences of 256 entries)
    g = np.load(GOLDEN / "viterbi.npz")
    X = torch.as_tensor(g[f"k{k}_Xfree"], dtype=torch.float32).cuda()
    assert np.array_equal(_viterbi_noalloc(lib, X, V, None, k).cpu().numpy(), g[f"k{k}_states_free"])
