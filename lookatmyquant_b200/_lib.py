"""ctypes bindings to liblamq_b200.so (the C ABI declared in include/lamq_b200.h).

The library is the product's only compute path: if it is missing or cannot load, every entry point raises — there is
no CPU or PyTorch fallback. `torch` tensors are passed as raw device pointers on the current CUDA stream.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "liblamq_b200.so"
_lib = None
_lock = threading.Lock()

LAMQ_OK, LAMQ_ERR_INVALID, LAMQ_ERR_CUDA, LAMQ_ERR_NOT_PD, LAMQ_ERR_TIMEOUT, LAMQ_ERR_NOT_PATH = range(6)
LAMQ_F32, LAMQ_BF16, LAMQ_F64 = 0, 1, 2

_c = ctypes
_P, _I64, _I32, _SZ, _D = _c.c_void_p, _c.c_int64, _c.c_int, _c.c_size_t, _c.c_double

# name -> (restype, argtypes): every symbol include/lamq_b200.h declares
SIGNATURES = {
    "lamq_abi_version": (_I32, []),
    "lamq_kernel_launches": (_c.c_uint64, []),
    "lamq_last_error": (_c.c_char_p, []),
    "lamq_viterbi_workspace_size": (_SZ, [_I64, _I32, _I32, _I32]),
    "lamq_viterbi": (_I32, [_P, _I64, _I32, _P, _I32, _I32, _P, _P, _P, _SZ, _P]),
    "lamq_viterbi_noalloc": (_I32, [_P, _I64, _I32, _P, _I32, _I32, _P, _P, _P]),
    "lamq_ldlq_round_workspace_size": (_SZ, [_I64]),
    "lamq_ldlq_round": (_I32, [_P, _I64, _I64, _I32, _P, _I64, _P, _I32, _I32, _P, _I64, _P, _SZ, _P]),
    "lamq_xtx_accumulate": (_I32, [_P, _I64, _P, _I64, _I64, _I32, _I32, _P, _I64, _I64, _P, _P]),
    "lamq_xtx_accumulate_scaled": (_I32, [_P, _I64, _P, _I64, _I64, _I32, _I32, _c.c_float, _P, _I64, _I64, _P, _P]),
    "lamq_gather_rows": (_I32, [_P, _I64, _P, _I64, _I32, _P, _P]),
    "lamq_weighted_split": (_I32, [_P, _I64, _P, _I64, _P, _P, _I64, _I32, _P, _P, _P]),
    "lamq_hessian_finalize": (_I32, [_P, _P, _I32, _I64, _D, _P, _P, _P]),
    "lamq_rht_rows": (_I32, [_P, _I64, _P, _I64, _I64, _I32, _I32, _P, _P, _P, _P, _D, _P]),
    "lamq_transpose_f64": (_I32, [_P, _I64, _P, _I64, _I32, _I32, _P]),
    "lamq_rht_rows_act": (_I32, [_P, _I32, _I64, _P, _I32, _I64, _I64, _I32, _I32, _P, _P, _P, _P, _D, _P]),
    "lamq_dgemm": (_I32, [_I32, _I32, _I32, _I32, _D, _P, _I64, _P, _I64, _D, _P, _I64, _P]),
    "lamq_factor_workspace_size": (_SZ, [_I32]),
    "lamq_cholesky_inverse_lower": (_I32, [_P, _I64, _I32, _P, _SZ, _P, _P]),
    "lamq_env_factor": (_I32, [_P, _I64, _I32, _D, _P, _I64, _P, _P, _SZ, _P, _P]),
    "lamq_ridge": (_I32, [_P, _I64, _P, _I64, _I32, _D, _P]),
    "lamq_cross_apply_workspace_size": (_SZ, [_I32, _I32]),
    "lamq_cross_apply": (_I32, [_P, _I64, _I32, _I32, _P, _I64, _P, _I64, _D, _P, _I64, _P, _SZ, _P]),
    "lamq_proxy_loss_workspace_size": (_SZ, [_I64, _I32]),
    "lamq_proxy_loss": (_I32, [_P, _I64, _P, _I64, _I64, _I32, _P, _I64, _P, _P, _P, _SZ, _P]),
    "lamq_trellis_words_per_row": (_I64, [_I32, _I32]),
    "lamq_kl_workspace_size": (_SZ, [_I64]),
    "lamq_kl_reference": (_I32, [_P, _I64, _I64, _I32, _P, _I64, _I32, _P, _I64, _P, _P, _P, _P, _SZ, _P, _P]),
    "lamq_kl_head": (_I32, [_P, _I64, _I64, _I32, _P, _I64, _I32, _P, _I64, _P, _P, _P, _P, _P, _P, _P, _SZ, _P, _P]),
    "lamq_ldlq_coltrellis_workspace_size": (_SZ, [_I64, _I32, _I32, _I32, _I32, _I32, _I32]),
    "lamq_ldlq_coltrellis": (_I32, [_P, _I64, _I64, _I32, _P, _I64, _P, _P, _P, _I32, _I32, _I32, _I32, _I32, _P, _P,
                                     _P, _SZ, _P]),
    "lamq_pack_trellis": (_I32, [_P, _I64, _I64, _I32, _I32, _I32, _P, _P, _P]),
    "lamq_unpack_trellis": (_I32, [_P, _I64, _I32, _I32, _I32, _P, _I64, _P]),
    "lamq_decode_trellis": (_I32, [_P, _I64, _I32, _I32, _I32, _P, _P, _P, _P, _I64, _P]),
    "lamq_trellis_product": (_I32, [_P, _I64, _I32, _I32, _I32, _P, _P, _P, _P, _I64, _I32, _P, _I64, _P]),
    "lamq_trellis_product_groups": (_I32, [_P, _I32, _I32, _P, _I64, _I32, _P]),
    "lamq_square_sums_workspace_size": (_SZ, [_I64, _I32]),
    "lamq_square_sums": (_I32, [_P, _I32, _I64, _I32, _I64, _P, _P, _P, _SZ, _P]),
    "lamq_trellis_gemm_workspace_size": (_SZ, [_P, _I32, _I64]),
    "lamq_trellis_gemm": (_I32, [_P, _I32, _I64, _I32, _P, _SZ, _P, _P]),
    "lamq_ldlq_rowtrellis_workspace_size": (_SZ, [_I64, _I32]),
    "lamq_ldlq_rowtrellis": (_I32, [_P, _I64, _I64, _I32, _P, _I64, _P, _P, _P, _P, _I32, _I32, _I32, _I32, _I32,
                                    _P, _P, _P, _SZ, _P]),
}


class ProductGroup(_c.Structure):
    """lamq_product_group: one packed row group of a grouped product (64 bytes, the header's field order)."""
    _fields_ = [("codes", _P), ("rows", _I64), ("k", _I32), ("L", _I32), ("scales", _P), ("table", _P),
                ("map", _P), ("y", _P), ("ldy", _I64)]


class GemmGroup(_c.Structure):
    """lamq_gemm_group: one row group of a trellis-dequant GEMM and its input (104 bytes, the header's field order)."""
    _fields_ = [("codes", _P), ("states", _P), ("lds", _I64), ("rows", _I64), ("k", _I32), ("L", _I32),
                ("scales", _P), ("table", _P), ("map", _P), ("y", _P), ("ldy", _I64), ("x", _P), ("ldx", _I64),
                ("n", _I32), ("reserved", _I32)]


class LamqError(RuntimeError):
    pass


def load():
    """Loads liblamq_b200.so (raising if it was not built) and declares every exported signature."""
    global _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise LamqError(f"{LIB_PATH} is missing: build it with `python -m lookatmyquant_b200.build` "
                                "(the CUDA kernels are the only implementation; there is no fallback)")
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                f = getattr(lib, name)
                f.restype, f.argtypes = res, args
            _lib = lib
    return _lib


def kernel_launches() -> int:
    """Kernels liblamq_b200 has launched in this process (lamq_kernel_launches)."""
    return int(load().lamq_kernel_launches())


def check(status: int, what: str):
    """Raises on a non-zero status."""
    if status != LAMQ_OK:
        msg = load().lamq_last_error().decode(errors="replace")
        if status == LAMQ_ERR_INVALID:
            raise ValueError(f"{what}: {msg}")
        if status == LAMQ_ERR_NOT_PD:
            raise AssertionError("H is not positive definite even with damping")
        if status == LAMQ_ERR_NOT_PATH:
            raise ValueError("the given projection is not a path through this trellis")
        raise LamqError(f"{what} failed (status {status}): {msg}")


def ptr(t) -> int | None:
    """Device pointer of a tensor (None for None)."""
    return None if t is None else t.data_ptr()


def stream_ptr(device=None) -> int:
    import torch
    return torch.cuda.current_stream(device).cuda_stream
