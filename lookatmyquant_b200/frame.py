"""The input environment of a linear core on B200: the host side of `opgraph.frame.Environment`
(ShinMegamiBoson/lookatmyquant, opgraph/frame.py:508-546)."""

from __future__ import annotations

import torch


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
        """tr(D H Dᵀ) (frame.py:532-535)."""
        D = D.double()
        H = self.H
        return float(torch.trace(D @ H @ D.T) if self.G is None else torch.trace(self.G @ D @ H @ D.T))
