"""The generic column sweep of the reference (`opgraph.syntax.sweep`) on the device, for any projection.

Reference: opgraph/syntax.py:86-124. Columns of W are settled `width` at a time; `on_block(j, T)` may look at the
running core T before each block of `block` columns; `project(j, columns, T)` returns the settled columns; with an
environment, Refit re-solves the later columns — lazily, as GPTQ does: inside a run of `lazy` columns every settled
block updates the rest of the run, and the columns after the run receive the run's accumulated update in one product.
Returns each column as it stood just before it was settled.

The order of the steps is the reference's, since the settled values depend on it; the run product T[:, b1:] −=
Z·U[b0:b1, b1:] runs on liblamq_b200's fp64 tensor-core GEMM when T is fp64 on a GPU. This is the path for arbitrary
Python projections (GPTQ and SparseGPT with width 1, vector codes); the trellis codes have fused kernels
(codes.ldlq_words: lamq_ldlq_rowtrellis, lamq_ldlq_coltrellis) that run whole sweeps in a few launches.
"""

from __future__ import annotations

from typing import Callable

import torch

from . import _lib
from ._lib import check, ptr, stream_ptr


def _run_update(T: torch.Tensor, Z: torch.Tensor, U: torch.Tensor, b0: int, b1: int):
    """T[:, b1:] −= Z·U[b0:b1, b1:]."""
    n = T.shape[1]
    if T.is_cuda and T.dtype == torch.float64 and T.stride(1) == 1:
        Uv = U if (U.dtype == torch.float64 and U.stride(1) == 1) else U.double().contiguous()
        Zc = Z.contiguous()
        src = Uv[b0:b1, b1:]
        dst = T[:, b1:]
        with torch.cuda.device(T.device):
            check(_lib.load().lamq_dgemm(0, T.shape[0], n - b1, b1 - b0, -1.0, ptr(Zc), Zc.stride(0), ptr(src),
                                         Uv.stride(0), 1.0, ptr(dst), T.stride(0), stream_ptr(T.device)), "lamq_dgemm")
    else:
        T[:, b1:] -= Z @ U[b0:b1, b1:].to(T.dtype)


def sweep(W: torch.Tensor, env, project: Callable[[int, torch.Tensor, torch.Tensor], torch.Tensor],
          block: int | None = None, on_block: Callable[[int, torch.Tensor], None] | None = None, width: int = 1,
          lazy: int = 128) -> torch.Tensor:
    """syntax.sweep: `env` is a frame.Environment (U, dead) or None; `project(j, cols, T)` gets the column itself
    when width is 1, else the width columns. Blocks chosen by on_block must not straddle a run."""
    T = W.clone()
    if env is not None:
        if lazy % width or (block and lazy % block):
            raise ValueError("lazy must be a multiple of width and of block")
        T[:, env.dead.to(T.device)] = 0
        U = env.U.to(T.device)
    before = torch.empty_like(T)
    rows, n = T.shape
    for b0 in range(0, n, lazy):
        b1 = min(b0 + lazy, n)
        Z = torch.empty(rows, b1 - b0, dtype=T.dtype, device=T.device)
        for j in range(b0, b1, width):
            if on_block is not None and block and j % block == 0:
                on_block(j, T)
            c1 = j + width
            before[:, j:c1] = T[:, j:c1]
            if width == 1:
                q = project(j, T[:, j], T)
                if env is None:
                    continue
                z = (T[:, j] - q) / U[j, j]  # E · U_jj⁻¹
                T[:, c1:b1] -= z[:, None] * U[j, c1:b1][None, :]
                Z[:, j - b0] = z
            else:
                q = project(j, T[:, j:c1], T)
                if env is None:
                    continue
                # z · U_BB = E for the upper-triangular diagonal block
                z = torch.linalg.solve_triangular(U[j:c1, j:c1], T[:, j:c1] - q, upper=True, left=False)
                T[:, c1:b1] -= z @ U[j:c1, c1:b1]
                Z[:, j - b0:j - b0 + width] = z
        if env is not None and b1 < n:
            _run_update(T, Z, U, b0, b1)
    return before
