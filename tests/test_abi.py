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
    st = lib.lamq_viterbi(None, 4, 8, None, 13, 2, None, None, None, 0, None)
    assert st == _lib.LAMQ_ERR_INVALID
    assert b"L must be 2..12" in lib.lamq_last_error()
    st = lib.lamq_ldlq_rowtrellis(None, 16, 4, 16, None, 16, None, None, None, None, 2, 12, 16, 20, 128,
                                  None, None, None, 0, None)
    assert st == _lib.LAMQ_ERR_INVALID
    assert lib.lamq_viterbi(None, 0, 8, None, 12, 2, None, None, None, 0, None) == _lib.LAMQ_OK  # empty input


def test_workspace_sizes(lib):
    assert lib.lamq_viterbi_workspace_size(100, 24, 12, 2) == 0  # short sequences keep back-pointers on chip
    # long sequences: the warp pair keeps them in shared memory where a device can hold them (0), else 256 B an entry
    assert lib.lamq_viterbi_workspace_size(3, 256, 12, 2) in (0, 3 * 256 * 32 * 8)
    assert lib.lamq_viterbi_workspace_size(2**60, 4096, 12, 2) in (0, 2**64 - 1)  # SIZE_MAX: the size overflows


# One call per entry point that breaks an argument rule: (name, arguments, a fragment of lamq_last_error()). Every
# entry point checks its arguments before it touches the device, so these run without a GPU.
N = None
P = 4096  # a non-null pointer the checks below never dereference
INVALID = [
    ("lamq_viterbi_noalloc", (P, 200000, 64, P, 12, 2, N, P, N), b"more back-pointers than the built-in"),
    ("lamq_viterbi_noalloc", (P, 2**62, 4096, P, 12, 2, N, P, N), b"more back-pointers than the built-in"),
    ("lamq_trellis_product", (P, 4, 32, 2, 12, P, P, N, P, 32, 2, P, 3, N), b"ldy 3 below the group's 4 rows"),
    ("lamq_viterbi_noalloc", (N, 4, 8, N, 12, 5, N, N, N), b"k must be 1..4"),
    ("lamq_ldlq_round", (N, 4, 4, 4, N, 4, N, 2, 200, N, 4, N, 0, N), b"block in 1..128"),
    ("lamq_ldlq_round", (N, 4, 4, 4, N, 4, N, 2, 16, N, 4, N, 0, N), b"null pointer"),
    ("lamq_xtx_accumulate", (N, 8, N, 8, -1, 8, 1, N, 8, 0, N, N), b"bad shape"),
    ("lamq_xtx_accumulate_scaled", (N, 8, N, 8, 16, 8, 1, 1.0, N, 8, 0, N, N), b"null pointer"),
    ("lamq_gather_rows", (N, 12, N, 4, 12, N, N), b"bad shape"),
    ("lamq_weighted_split", (N, 8, N, 8, N, N, 4, 0, N, N, N), b"bad shape"),
    ("lamq_hessian_finalize", (N, N, 4, 4, 0.0, N, N, N), b"bad shape"),
    ("lamq_hessian_finalize", (N, N, 4, 4, 1.0, N, N, N), b"null pointer"),
    ("lamq_rht_rows", (N, 4, N, 4, 2, 0, 4, N, N, N, N, 1.0, N), b"factor orders"),
    ("lamq_transpose_f64", (N, 4, N, 4, -1, 4, N), b"negative shape"),
    ("lamq_rht_rows_act", (N, 1, 4, N, 1, 4, 2, 0, 4, N, N, N, N, 1.0, N), b"factor orders"),
    ("lamq_rht_rows_act", (N, 5, 4, N, 1, 4, 2, 2, 2, N, N, N, N, 1.0, N), b"input dtype"),
    ("lamq_rht_rows_act", (P, 1, 4, P, 1, 4, 2, 2, 2, P, P, N, N, 1.0, N), b"must not alias"),
    ("lamq_dgemm", (0, -1, 4, 4, 1.0, N, 4, N, 4, 0.0, N, 4, N), b"negative shape"),
    ("lamq_dgemm", (0, 4, 4, 4, 1.0, N, 4, N, 4, 0.0, N, 4, N), b"null pointer"),
    ("lamq_cholesky_inverse_lower", (N, 2, 4, N, 0, N, N), b"bad shape"),
    ("lamq_env_factor", (N, 4, 4, 0.01, N, 4, N, N, 0, N, N), b"null or aliased"),
    ("lamq_ridge", (N, 2, N, 4, 4, 0.1, N), b"bad shape"),
    ("lamq_proxy_loss", (N, 2, N, 4, 4, 4, N, 4, N, N, N, 0, N), b"bad shape"),
    ("lamq_square_sums", (N, 0, 4, 8, 4, N, N, N, 0, N), b"bad shape"),
    ("lamq_square_sums", (N, 2, 4, 8, 8, N, N, N, 0, N), b"dtype"),
    ("lamq_square_sums", (P, 0, 4, 8, 8, P, N, N, 0, N), b"workspace"),
    ("lamq_proxy_loss", (N, 4, N, 4, 4, 4, N, 4, N, P, N, 0, N), b"null pointer"),
    ("lamq_cross_apply", (N, 4, 6, 4, N, 4, N, 4, 0.5, N, 4, N, 0, N), b"needs rows == n"),
    ("lamq_kl_reference", (N, 8, 0, 8, N, 8, 16, N, 16, N, N, N, N, 0, N, N), b"lamq_kl_reference: bad shape"),
    ("lamq_kl_head", (N, 8, 4, 8, N, 8, 16, N, 16, N, N, N, N, N, N, N, 0, N, N), b"lamq_kl_head: null pointer"),
    ("lamq_ldlq_coltrellis", (N, 8, 8, 8, N, 8, N, N, N, 2, 11, 8, 1, 8, N, N, N, 0, N), b"L = 12"),
    ("lamq_ldlq_coltrellis", (N, 8, 12, 8, N, 8, N, N, N, 2, 12, 8, 1, 8, N, N, N, 0, N), b"multiple of the run"),
    ("lamq_pack_trellis", (N, 32, 4, 32, 0, 12, N, N, N), b"unsupported widths"),
    ("lamq_unpack_trellis", (N, 4, 32, 2, 13, N, 32, N), b"unsupported widths"),
    ("lamq_decode_trellis", (N, 4, 32, 2, 12, N, N, N, N, 16, N), b"leading dimension"),
    ("lamq_trellis_product", (N, 4, 32, 2, 12, N, N, N, N, 32, -1, N, 4, N), b"bad vector shape"),
    ("lamq_trellis_product_groups", (N, 1, 0, N, 32, 1, N), b"bad shape"),
    ("lamq_trellis_product_groups", (N, 1, 32, N, 32, 1, N), b"null pointer"),
    ("lamq_trellis_gemm", (N, 1, -1, 0, N, 0, N, N), b"bad shape"),
    ("lamq_trellis_gemm", (N, 1, 64, 0, N, 0, N, N), b"null pointer"),
]

# Empty inputs are a successful no-op, as the reference's loops over no rows are.
EMPTY = [
    ("lamq_viterbi_noalloc", (N, 0, 8, N, 12, 2, N, N, N)),
    ("lamq_ldlq_round", (N, 4, 0, 4, N, 4, N, 2, 16, N, 4, N, 0, N)),
    ("lamq_ldlq_rowtrellis", (N, 16, 0, 16, N, 16, N, N, N, N, 2, 12, 16, 20, 128, N, N, N, 0, N)),
    ("lamq_xtx_accumulate", (N, 8, N, 8, 0, 8, 1, N, 8, 0, N, N)),
    ("lamq_gather_rows", (N, 8, N, 0, 8, N, N)),
    ("lamq_weighted_split", (N, 8, N, 8, N, N, 0, 8, N, N, N)),
    ("lamq_rht_rows", (N, 4, N, 4, 0, 2, 2, N, N, N, N, 1.0, N)),
    ("lamq_transpose_f64", (N, 4, N, 4, 0, 4, N)),
    ("lamq_rht_rows_act", (N, 1, 4, N, 1, 4, 0, 2, 2, N, N, N, N, 1.0, N)),
    ("lamq_dgemm", (0, 0, 4, 4, 1.0, N, 4, N, 4, 0.0, N, 4, N)),
    ("lamq_cholesky_inverse_lower", (N, 0, 0, N, 0, N, N)),
    ("lamq_env_factor", (N, 0, 0, 0.01, N, 0, N, N, 0, N, N)),
    ("lamq_ridge", (N, 0, N, 0, 0, 0.1, N)),
    ("lamq_proxy_loss", (N, 4, N, 4, 4, 0, N, 4, N, P, N, 0, N)),
    ("lamq_square_sums", (N, 1, 0, 8, 8, N, N, N, 0, N)),
    ("lamq_cross_apply", (N, 4, 0, 0, N, 4, N, 4, 0.5, N, 4, N, 0, N)),
    ("lamq_pack_trellis", (N, 32, 0, 32, 2, 12, N, N, N)),
    ("lamq_unpack_trellis", (N, 0, 32, 2, 12, N, 32, N)),
    ("lamq_decode_trellis", (N, 0, 32, 2, 12, N, N, N, N, 32, N)),
    ("lamq_trellis_product", (N, 4, 32, 2, 12, N, N, N, N, 32, 0, N, 4, N)),
    ("lamq_trellis_product_groups", (N, 0, 32, N, 32, 1, N)),
    ("lamq_trellis_gemm", (N, 0, 64, 0, N, 0, N, N)),
    ("lamq_trellis_gemm", (P, 1, 0, 0, N, 0, P, N)),
]


@pytest.mark.parametrize("name,args,text", INVALID, ids=[f"{c[0]}-{i}" for i, c in enumerate(INVALID)])
def test_entry_point_rejects_bad_arguments(lib, name, args, text):
    before = lib.lamq_kernel_launches()
    assert getattr(lib, name)(*args) == _lib.LAMQ_ERR_INVALID
    assert text in lib.lamq_last_error()
    assert lib.lamq_kernel_launches() == before


@pytest.mark.parametrize("name,args", EMPTY, ids=[c[0] for c in EMPTY])
def test_entry_point_accepts_empty_input(lib, name, args):
    before = lib.lamq_kernel_launches()
    assert getattr(lib, name)(*args) == _lib.LAMQ_OK
    assert lib.lamq_kernel_launches() == before


def test_invalid_and_empty_tables_cover_every_compute_entry_point():
    compute = {n for n in declared() if not n.endswith(("_workspace_size", "_words_per_row"))}
    compute -= {"lamq_abi_version", "lamq_last_error", "lamq_kernel_launches"}
    covered = {c[0] for c in INVALID} | {c[0] for c in EMPTY} | {"lamq_viterbi", "lamq_ldlq_rowtrellis"}
    assert compute <= covered, sorted(compute - covered)


def test_product_group_layout_matches_the_header(lib):
    """The ctypes lamq_product_group reaches the library field for field: the checks quote rows, k and L back."""
    assert ctypes.sizeof(_lib.ProductGroup) == 64
    x = ctypes.c_float(0.0)
    bad = [_lib.ProductGroup(None, 0, 1, 12, None, None, None, None, 0),
           _lib.ProductGroup(None, -7, 1, 12, None, None, None, None, 0)]
    arr = (_lib.ProductGroup * 2)(*bad)
    assert lib.lamq_trellis_product_groups(arr, 2, 32, ctypes.addressof(x), 32, 1, None) == _lib.LAMQ_ERR_INVALID
    assert b"group 1 has -7 rows" in lib.lamq_last_error()
    arr[1] = _lib.ProductGroup(None, 4, 5, 11, None, None, None, None, 0)
    assert lib.lamq_trellis_product_groups(arr, 2, 32, ctypes.addressof(x), 32, 1, None) == _lib.LAMQ_ERR_INVALID
    assert b"group 1: widths" in lib.lamq_last_error() and b"(k 5, L 11)" in lib.lamq_last_error()
    arr[1] = _lib.ProductGroup(None, 4, 3, 12, None, None, None, None, 0)
    assert lib.lamq_trellis_product_groups(arr, 2, 32, ctypes.addressof(x), 32, 1, None) == _lib.LAMQ_ERR_INVALID
    assert b"group 1: null pointer" in lib.lamq_last_error()


def test_gemm_group_layout_matches_the_header(lib):
    """The ctypes lamq_gemm_group reaches the library field for field: the checks quote rows, n, k and L back."""
    assert ctypes.sizeof(_lib.GemmGroup) == 104
    st = ctypes.c_int(0)

    def grp(codes, states, lds, rows, k, L, x=P + 16, ldx=16, n=16):
        return _lib.GemmGroup(codes, states, lds, rows, k, L, P, P, None, P, max(rows, 4), x, ldx, n, 0)
    arr = (_lib.GemmGroup * 2)(grp(None, None, 0, 0, 1, 12), grp(None, None, 0, -3, 1, 12))
    assert lib.lamq_trellis_gemm(arr, 2, 1, 0, None, 0, ctypes.addressof(st), None) == _lib.LAMQ_ERR_INVALID
    assert b"group 1 has -3 rows" in lib.lamq_last_error()
    arr[1] = grp(P, None, 0, 4, 5, 12)
    assert lib.lamq_trellis_gemm(arr, 2, 1, 0, None, 0, ctypes.addressof(st), None) == _lib.LAMQ_ERR_INVALID
    assert b"group 1: packed widths" in lib.lamq_last_error() and b"(k 5, L 12)" in lib.lamq_last_error()
    arr[1] = grp(P, P, 16, 4, 2, 12)
    assert lib.lamq_trellis_gemm(arr, 2, 1, 0, None, 0, ctypes.addressof(st), None) == _lib.LAMQ_ERR_INVALID
    assert b"not both" in lib.lamq_last_error()
    arr[1] = grp(P, None, 0, 4, 2, 12, x=P + 8)
    assert lib.lamq_trellis_gemm(arr, 2, 1, 0, None, 0, ctypes.addressof(st), None) == _lib.LAMQ_ERR_INVALID
    assert b"16-byte aligned" in lib.lamq_last_error()
    arr[1] = grp(P, None, 0, 4, 2, 12, ldx=8, n=16)
    assert lib.lamq_trellis_gemm(arr, 2, 1, 0, None, 0, ctypes.addressof(st), None) == _lib.LAMQ_ERR_INVALID
    assert b"bad input shape (n 16, ldx 8)" in lib.lamq_last_error()
    # from 513 vectors the weights are decoded once into a workspace of rows x ceil(n / 8)·8 bf16
    arr[0] = grp(P, None, 0, 300, 2, 12, n=100, ldx=104)
    arr[1] = grp(P, None, 0, 0, 2, 12)
    assert lib.lamq_trellis_gemm_workspace_size(arr, 2, 512) == 0
    assert lib.lamq_trellis_gemm_workspace_size(arr, 2, 513) == 300 * 104 * 2
    assert lib.lamq_trellis_gemm(arr, 2, 513, 0, None, 0, ctypes.addressof(st), None) == _lib.LAMQ_ERR_INVALID
    assert b"workspace of 62400 bytes" in lib.lamq_last_error()
