"""Scalar-level LDLQ on B200 in fp64: the reference's `opgraph.ldlq_gpu` module (used by nested.py:117-119 to round a
matrix to a fixed set of levels, GPTQ's lazy-batch form), on liblamq_b200's kernels.

    U = ldlq_factor(Hr)                 # once per input statistics (H in the rotated basis)
    Q = ldlq_round(X, U, levels)        # X: rows in units of their RMS; returns the chosen levels

Reference: opgraph/ldlq_gpu.py:15-26 (`ldlq_factor`: H symmetrized, damping d·mean(diag H)·I with d = damp, 10·damp,
100·damp until H factors, U the upper Cholesky factor of H⁻¹) and :29-49 (`ldlq_round`). Here U comes from
lamq_env_factor (one Cholesky of the flipped matrix and one triangular inverse, the same unique factor) and the
rounding from lamq_ldlq_round (a thread per row inside each block, the reference's separately rounded fp64 operations,
the product after each block on the fp64 tensor cores).
"""

from __future__ import annotations

import torch

from . import _lib
from ._lib import check, ptr, stream_ptr


def _dev_f64(M: torch.Tensor, device=None) -> torch.Tensor:
    dev = torch.device(device) if device is not None else (M.device if M.is_cuda else torch.device("cuda"))
    return M.to(dev, torch.float64).contiguous()


def ldlq_factor(Hr: torch.Tensor, damp: float = 0.01) -> torch.Tensor:
    """The upper Cholesky factor of (H + d·mean(diag H)·I)⁻¹ for the first d in (damp, 10·damp, 100·damp) at which
    the symmetrized H factors (fp64, on the GPU). Raises AssertionError, as the reference does, when none does."""
    from .linalg import env_factor
    H = _dev_f64(Hr)
    H = 0.5 * (H + H.T)
    eye = torch.eye(H.shape[0], dtype=H.dtype, device=H.device)
    mean = H.diagonal().mean()
    for d in (damp, 10 * damp, 100 * damp):
        status = torch.zeros(1, dtype=torch.int32, device=H.device)
        U, _, _ = env_factor(H + d * mean * eye, 0.0, status=status)
        if int(status.item()) == 0:
            return U
    raise AssertionError("H is not positive definite even with damping")


@torch.no_grad()
def ldlq_round(X: torch.Tensor, U: torch.Tensor, levels: torch.Tensor, block: int = 128) -> torch.Tensor:
    """Each entry of X (rows × inputs) to one of the sorted `levels`, inputs in order, each rounding error carried into
    the later inputs through U (blocks of `block` <= 128 inputs). Returns the chosen levels (fp64, on the GPU)."""
    if not 1 <= block <= 128:
        raise ValueError("block must be in 1..128")
    Xw = _dev_f64(X).clone()
    dev = Xw.device
    Ud = _dev_f64(U, dev)
    lv = _dev_f64(levels.reshape(-1), dev)
    rows, n = Xw.shape
    if Ud.shape != (n, n):
        raise ValueError(f"U is {tuple(Ud.shape)}, X has {n} inputs")
    Q = torch.empty_like(Xw)
    lib = _lib.load()
    ws = torch.empty(max(lib.lamq_ldlq_round_workspace_size(rows), 1), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        check(lib.lamq_ldlq_round(ptr(Xw), Xw.stride(0), rows, n, ptr(Ud), Ud.stride(0), ptr(lv), lv.numel(), block,
                                  ptr(Q), Q.stride(0), ptr(ws), ws.numel(), stream_ptr(dev)), "lamq_ldlq_round")
    return Q
