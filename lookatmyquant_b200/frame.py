"""The input environment of a linear core on B200: the host side of `opgraph.frame.Environment`
(ShinMegamiBoson/lookatmyquant, opgraph/frame.py:508-546)."""

from __future__ import annotations

import torch

from . import _lib
from ._lib import check, ptr, stream_ptr


def proxy_loss(Wq: torch.Tensor, W: torch.Tensor | None, H: torch.Tensor, per_row: bool = False):
    """The proxy loss tr(E·H·Eᵀ) = Σ (E @ H) ⊙ E with E = Wq − W (W None: E = Wq), as best_word scores a word
    (quantize.py:1320-1325), on the device in fp64 (lamq_proxy_loss: E·H on the fp64 tensor cores, a fixed-order sum).
    Returns a 0-d fp64 device tensor (and the per-row losses with `per_row`); nothing is read back to the host."""
    if not Wq.is_cuda:
        raise RuntimeError("proxy_loss expects CUDA tensors")
    dev = Wq.device
    Wq = Wq.to(torch.float64)
    Wq = Wq if Wq.stride(-1) == 1 else Wq.contiguous()
    rows, n = Wq.shape
    if W is not None:
        W = W.to(dev, torch.float64)
        W = W if W.stride(-1) == 1 else W.contiguous()
        if W.shape != Wq.shape:
            raise ValueError(f"word {tuple(Wq.shape)} and target {tuple(W.shape)} differ in shape")
    H = H.to(dev, torch.float64)
    H = H if H.stride(-1) == 1 else H.contiguous()
    if H.shape != (n, n):
        raise ValueError(f"H is {tuple(H.shape)}, the word has {n} inputs")
    lib = _lib.load()
    total = torch.zeros((), dtype=torch.float64, device=dev)
    rl = torch.zeros(rows, dtype=torch.float64, device=dev) if per_row else None
    ws = torch.empty(max(lib.lamq_proxy_loss_workspace_size(rows, n), 1), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        check(lib.lamq_proxy_loss(ptr(Wq), Wq.stride(0), ptr(W), 0 if W is None else W.stride(0), rows, n, ptr(H),
                                  H.stride(0), ptr(rl), ptr(total), ptr(ws), ws.numel(), stream_ptr(dev)),
              "lamq_proxy_loss")
    return (total, rl) if per_row else total


class Environment:
    """What the rest of the network sees through a linear core's input bond: H = Σ x xᵀ, damped (frame.py:508-522).

    `U` is the upper Cholesky factor of H⁻¹ (its rows are the Schur-complement updates of Refit); `dead` flags inputs
    with a zero diagonal, which get a unit diagonal before damping. Computed on H's CUDA device in fp64 by
    lamq_env_factor (U = J·chol(J·H·J)⁻¹·J on the fp64 tensor cores). `check()` raises the reference's error when H was
    not positive definite; it synchronises, so callers run it once the factor is needed on the host.
    """

    def __init__(self, H: torch.Tensor, damp: float = 0.01, G: torch.Tensor | None = None,
                 status: torch.Tensor | None = None):
        from .linalg import env_factor
        if not H.is_cuda:
            raise RuntimeError("Environment expects H on a CUDA device")
        self.G = None if G is None else G.double()
        self._H0, self.damp = H.double(), damp
        self.U, self.dead, self.check = env_factor(self._H0, damp, status)

    @classmethod
    def from_factor(cls, H, U: torch.Tensor, dead: torch.Tensor, status: torch.Tensor,
                    damp: float = 0.01) -> "Environment":
        """An environment whose factor was computed elsewhere (another rank): U, the dead flags and the status word
        of that factorization. `H` is the matrix or a zero-argument callable that forms it (only `H`/`error` use it,
        so a rank that only sweeps never forms it)."""
        from .linalg import status_check
        env = cls.__new__(cls)
        env.G, env._H0, env.damp = None, H if callable(H) else H.double(), damp
        env.U, env.dead, env.check = U, dead.bool(), status_check(status)
        return env

    @property
    def H(self) -> torch.Tensor:
        """The damped H (frame.py:517-521)."""
        if callable(self._H0):
            self._H0 = self._H0().double()
        H = self._H0.clone()
        idx = torch.nonzero(self.dead).flatten()
        H[idx, idx] = 1
        return H + self.damp * torch.mean(torch.diag(H)) * torch.eye(len(H), dtype=H.dtype, device=H.device)

    def error(self, D: torch.Tensor) -> float:
        """tr(D H Dᵀ) (frame.py:532-535), on the device (lamq_proxy_loss)."""
        if self.G is not None:
            raise NotImplementedError("output-weighted (G) errors are not on the B200 path")
        return float(proxy_loss(D.to(self.U.device), None, self.H).item())
