"""The input environment of a linear core on B200: the host side of `opgraph.frame.Environment`
(ShinMegamiBoson/lookatmyquant, opgraph/frame.py:508-546)."""

from __future__ import annotations

import torch


class Environment:
    """What the rest of the network sees through a linear core's input bond: H = Σ x xᵀ, damped (frame.py:508-522).

    `U` is the upper Cholesky factor of H⁻¹ (its rows are the Schur-complement updates of Refit); `dead` flags inputs
    with a zero diagonal, which get a unit diagonal before damping. Everything stays on H's CUDA device in fp64.
    """

    def __init__(self, H: torch.Tensor, damp: float = 0.01, G: torch.Tensor | None = None):
        if not H.is_cuda:
            raise RuntimeError("Environment expects H on a CUDA device")
        self.G = None if G is None else G.double()
        H = H.clone().double()
        self.dead = torch.diag(H) == 0
        idx = torch.nonzero(self.dead).flatten()
        H[idx, idx] = 1
        H += damp * torch.mean(torch.diag(H)) * torch.eye(len(H), dtype=H.dtype, device=H.device)
        self.H = H
        self.U = torch.linalg.cholesky(torch.cholesky_inverse(torch.linalg.cholesky(H)), upper=True).contiguous()

    def error(self, D: torch.Tensor) -> float:
        """tr(D H Dᵀ) (frame.py:532-535)."""
        D = D.double()
        return float(torch.trace(D @ self.H @ D.T) if self.G is None else torch.trace(self.G @ D @ self.H @ D.T))
