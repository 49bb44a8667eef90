"""fp64 dense linear algebra of the build on the fp64 tensor cores (liblamq_b200: lamq_dgemm, lamq_env_factor,
lamq_cholesky_inverse_lower, lamq_ridge).

Reference: opgraph/frame.py:515-522 (`Environment`: U = chol(cholesky_inverse(chol(H)))ᵀ after dead inputs and
damping) and quantize.py:1330-1335 (`cross_target`: M = I + α·(solve(H + λ·mean(diag H)·I, Dᵀ))ᵀ), torch.linalg in
fp64 there. Here U = J·chol(J·H·J)⁻¹·J (the same unique factor) and the QEP target W·M is formed through the Cholesky
factor of H + λ·mean(diag H)·I: W·M = W + α·((W·D)·Lc⁻ᵀ)·Lc⁻¹.
"""

from __future__ import annotations

import torch

from . import _lib
from ._lib import check, ptr, stream_ptr


def _f64(M: torch.Tensor) -> torch.Tensor:
    if M.dtype != torch.float64 or not M.is_cuda:
        raise TypeError("fp64 CUDA tensors expected")
    return M if M.stride(-1) == 1 else M.contiguous()


def _status(dev):
    return torch.zeros(1, dtype=torch.int32, device=dev)


def _raise_if_not_pd(status):
    if int(status.item()) == _lib.LAMQ_ERR_NOT_PD:
        raise AssertionError("H is not positive definite even with damping")
    _lib.check(int(status.item()), "factorization")


def gemm(A, B, C=None, transB=False, alpha=1.0, beta=0.0):
    """C = α·A·B (or α·A·Bᵀ) + β·C, fp64 on the tensor cores."""
    A, B = _f64(A), _f64(B)
    M, K = A.shape
    N = B.shape[0] if transB else B.shape[1]
    if C is None:
        C = torch.empty(M, N, dtype=torch.float64, device=A.device)
        beta = 0.0
    with torch.cuda.device(A.device):
        check(_lib.load().lamq_dgemm(1 if transB else 0, M, N, K, float(alpha), ptr(A), A.stride(0), ptr(B),
                                     B.stride(0), float(beta), ptr(C), C.stride(0), stream_ptr(A.device)),
              "lamq_dgemm")
    return C


def env_factor(H: torch.Tensor, damp: float = 0.01, status: torch.Tensor | None = None):
    """(U, dead, check): the environment factor of frame.py:515-522 on the GPU. `check()` raises the reference's
    error if H was not positive definite (it synchronises; call it when the result is needed)."""
    H = _f64(H)
    n = H.shape[0]
    dev = H.device
    lib = _lib.load()
    U = torch.empty(n, n, dtype=torch.float64, device=dev)
    dead = torch.empty(n, dtype=torch.uint8, device=dev)
    ws = torch.empty(lib.lamq_factor_workspace_size(n), dtype=torch.uint8, device=dev)
    st = _status(dev) if status is None else status
    with torch.cuda.device(dev):
        check(lib.lamq_env_factor(ptr(H), H.stride(0), n, float(damp), ptr(U), n, ptr(dead), ptr(ws), ws.numel(),
                                  ptr(st), stream_ptr(dev)), "lamq_env_factor")
    return U, dead.bool(), lambda: _raise_if_not_pd(st)


def status_check(st: torch.Tensor):
    """The deferred check of a factorization's status word (as env_factor and cholesky_inverse_lower return)."""
    return lambda: _raise_if_not_pd(st)


def cholesky_inverse_lower(A: torch.Tensor, deferred: bool = False, status: torch.Tensor | None = None):
    """L⁻¹ for A = L·Lᵀ (lower triangular, fp64), on a copy of A. With `deferred`, returns (L⁻¹, check) and leaves the
    positive-definiteness check (a synchronisation) to the caller."""
    A = _f64(A).clone()
    n = A.shape[0]
    lib = _lib.load()
    ws = torch.empty(lib.lamq_factor_workspace_size(n), dtype=torch.uint8, device=A.device)
    st = _status(A.device) if status is None else status
    with torch.cuda.device(A.device):
        check(lib.lamq_cholesky_inverse_lower(ptr(A), A.stride(0), n, ptr(ws), ws.numel(), ptr(st),
                                              stream_ptr(A.device)), "lamq_cholesky_inverse_lower")
    if deferred:
        return A, lambda: _raise_if_not_pd(st)
    _raise_if_not_pd(st)
    return A


def ridge(H: torch.Tensor, lam: float) -> torch.Tensor:
    """H + λ·mean(diag H)·I."""
    H = _f64(H)
    n = H.shape[0]
    A = torch.empty_like(H)
    with torch.cuda.device(H.device):
        check(_lib.load().lamq_ridge(ptr(H), H.stride(0), ptr(A), n, n, float(lam), stream_ptr(H.device)),
              "lamq_ridge")
    return A


class CrossTarget:
    """The QEP map of quantize.py:1330-1335 for one stage: `apply(W)` = W·M with M = I + α·(solve(H + λ·mean(diag H)·I,
    Dᵀ))ᵀ = I + α·D·(H + λμI)⁻¹ (lamq_cross_apply). With `rows` (the rows the stage will map) above n, M is formed
    once; otherwise each W is mapped as W + α·((W·D)·Lc⁻ᵀ)·Lc⁻¹."""

    def __init__(self, H, D, alpha: float, lam: float, rows: int | None = None, Linv=None, check=None):
        n = H.shape[0] if H is not None else D.shape[0]
        self.alpha = alpha
        if Linv is None:
            self.Linv, self.check = cholesky_inverse_lower(ridge(H, lam), deferred=True)
        else:  # the factor computed elsewhere (another rank)
            self.Linv, self.check = _f64(Linv), (check or (lambda: None))
        self.D = _f64(D)
        self.M = None
        if rows is None or rows > n:
            self.M = self._apply(None, n)

    def record_stream(self, stream):
        """Marks the map's tensors as used on `stream` (they were made on another stream)."""
        for t in (self.Linv, self.D, self.M):
            if t is not None:
                t.record_stream(stream)

    def _apply(self, W, rows):
        n = self.D.shape[0]
        dev = self.D.device
        lib = _lib.load()
        out = torch.empty(rows, n, dtype=torch.float64, device=dev)
        ws = torch.empty(lib.lamq_cross_apply_workspace_size(rows, n), dtype=torch.uint8, device=dev)
        with torch.cuda.device(dev):
            check(lib.lamq_cross_apply(ptr(W), 0 if W is None else W.stride(0), rows, n, ptr(self.D),
                                       self.D.stride(0), ptr(self.Linv), self.Linv.stride(0), float(self.alpha),
                                       ptr(out), n, ptr(ws), ws.numel(), stream_ptr(dev)), "lamq_cross_apply")
        return out

    def apply(self, W: torch.Tensor) -> torch.Tensor:
        W = _f64(W)
        if self.M is not None:
            return gemm(W, self.M)
        return self._apply(W, W.shape[0])
