"""Randomized Hadamard rotations applied through their Kronecker factors (liblamq_b200 lamq_rht_rows).

Reference: opgraph/codes.py:97-132 (`hadamard_factors`, `hadamard`, `rht`): R = (A ⊗ B)/√n · diag(s) with A a
Sylvester and B a Sylvester or Paley ±1 matrix, s random signs from torch's CPU generator (codes.py:131). The
reference forms R densely and multiplies; here R is never formed: each row is transformed as A·V·Bᵀ in one kernel.
"""

from __future__ import annotations

import math

import torch

from . import _lib
from ._lib import check, ptr, stream_ptr


def _sign_bits(M: torch.Tensor) -> torch.Tensor:
    """Row-wise sign bits of a ±1 matrix: word w of row p has bit k set when M[p][32w + k] < 0 (int32 words)."""
    rows, cols = M.shape
    words = (cols + 31) // 32
    neg = torch.zeros(rows, words * 32, dtype=torch.int64)
    neg[:, :cols] = (M < 0).to(torch.int64)
    weights = (1 << torch.arange(32, dtype=torch.int64))
    packed = (neg.reshape(rows, words, 32) * weights).sum(-1)
    return packed.to(torch.uint32).view(torch.int32) if hasattr(torch, "uint32") else packed.to(torch.int32)


class Rotation:
    """rht(n, seed) held as its factors and signs on a device. `rows(M)` = M·Rᵀ (R applied to each row),
    `rows_t(M)` = M·R (Rᵀ applied to each row), `conj(H)` = R·H·Rᵀ for symmetric H."""

    def __init__(self, n: int, seed: int, device=None):
        from .codes import hadamard_factors, rht_signs
        dev = torch.device(device or "cuda")
        A, B = hadamard_factors(n)
        self.n, self.seed, self.device = n, seed, dev
        self.a, self.b = A.shape[0], B.shape[0]
        self.scale = 1.0 / math.sqrt(n)
        self.signs = rht_signs(n, seed).to(dev)
        self.Abits, self.Bbits = _sign_bits(A).to(dev), _sign_bits(B).to(dev)
        self.Atbits, self.Btbits = _sign_bits(A.T.contiguous()).to(dev), _sign_bits(B.T.contiguous()).to(dev)

    @classmethod
    def from_signs(cls, signs: torch.Tensor, device=None) -> "Rotation":
        """The rotation of a stored `.signs` vector (±1, compiler_artifact.py:300-304) instead of a seed."""
        rot = cls(int(signs.numel()), 0, device)
        rot.seed = None
        rot.signs = signs.reshape(-1).to(rot.device, torch.float64)
        return rot

    def _run(self, M, out, transpose: bool):
        if M.dtype != torch.float64 or not M.is_cuda:
            raise TypeError("rotations run on fp64 CUDA tensors")
        M = M if M.stride(-1) == 1 else M.contiguous()
        rows = M.shape[0]
        if M.shape[1] != self.n:
            raise ValueError(f"rows of length {M.shape[1]}, rotation of order {self.n}")
        out = torch.empty_like(M, memory_format=torch.contiguous_format) if out is None else out
        ab, bb = (self.Atbits, self.Btbits) if transpose else (self.Abits, self.Bbits)
        pre, post = (None, self.signs) if transpose else (self.signs, None)
        with torch.cuda.device(self.device):
            check(_lib.load().lamq_rht_rows(ptr(M), M.stride(0), ptr(out), out.stride(0), rows, self.a, self.b,
                                            ptr(ab), ptr(bb), ptr(pre), ptr(post), self.scale,
                                            stream_ptr(self.device)), "lamq_rht_rows")
        return out

    def _act(self, X, transpose: bool, out_dtype):
        """lamq_rht_rows_act: the rotation of activation rows (bf16/fp32/fp64 in, fp32 sums, bf16/fp32 out)."""
        if not X.is_cuda:
            raise TypeError("rotations run on CUDA tensors")
        dt = {torch.bfloat16: _lib.LAMQ_BF16, torch.float32: _lib.LAMQ_F32, torch.float64: _lib.LAMQ_F64}
        if X.dtype not in dt or out_dtype not in (torch.bfloat16, torch.float32):
            raise TypeError(f"activation rotation: {X.dtype} in, {out_dtype} out not supported")
        X = X.reshape(-1, X.shape[-1])
        X = X if X.stride(-1) == 1 else X.contiguous()
        if X.shape[1] != self.n:
            raise ValueError(f"rows of length {X.shape[1]}, rotation of order {self.n}")
        rows = X.shape[0]
        ld = (self.n + 7) // 8 * 8  # 16-byte rows: the bf16 output is a TMA operand
        out = torch.empty(rows, ld, dtype=out_dtype, device=X.device)[:, :self.n]
        ab, bb = (self.Atbits, self.Btbits) if transpose else (self.Abits, self.Bbits)
        pre, post = (None, self.signs) if transpose else (self.signs, None)
        with torch.cuda.device(self.device):
            check(_lib.load().lamq_rht_rows_act(ptr(X), dt[X.dtype], X.stride(0), ptr(out), dt[out_dtype],
                                                out.stride(0), rows, self.a, self.b, ptr(ab), ptr(bb), ptr(pre),
                                                ptr(post), self.scale, stream_ptr(self.device)),
                  "lamq_rht_rows_act")
        return out

    def rows_act(self, X: torch.Tensor, out_dtype=torch.bfloat16) -> torch.Tensor:
        """X·Rᵀ for activation rows (R applied to each row), summed in fp32, as bf16 (a tensor-core operand with
        16-byte rows) or fp32."""
        return self._act(X, False, out_dtype)

    def rows_t_act(self, X: torch.Tensor, out_dtype=torch.bfloat16) -> torch.Tensor:
        """X·R for activation rows (Rᵀ applied to each row), summed in fp32."""
        return self._act(X, True, out_dtype)

    def rows(self, M: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """M·Rᵀ: X = W·R_inᵀ (codes.py:430)."""
        return self._run(M, out, False)

    def rows_t(self, M: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """M·R: the dequantized W_q = (S ⊙ V)·R_in."""
        return self._run(M, out, True)

    def conj(self, H: torch.Tensor) -> torch.Tensor:
        """R·H·Rᵀ for symmetric H (codes.py:439): rows of H, a transpose, rows again."""
        G = self.rows(H)
        Gt = torch.empty_like(G)
        with torch.cuda.device(self.device):
            check(_lib.load().lamq_transpose_f64(ptr(G), G.stride(0), ptr(Gt), Gt.stride(0), self.n, self.n,
                                                 stream_ptr(self.device)), "lamq_transpose_f64")
        return self.rows(Gt, out=G)
