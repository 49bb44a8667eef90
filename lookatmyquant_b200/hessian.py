"""Input statistics on B200: the token-weighted Hessian H and the QEP cross moment D.

Reference: quantize.py:1412-1470 (inside `quantize_stage`): for every calibration chunk of activations X (the
quantized stream) and X_ref (the reference stream), with per-token weights w of mean 1,

    H += Xᵀ (w ⊙ X),   D += X_refᵀ (w ⊙ X),   n_tok += tokens        (fp32, on the GPU)
    H = H / n_tok (fp64),   D = D / n_tok − H (fp64)

and compiler.py:233-265 (`capture`), the unweighted H of the `measure` sweep. Here the contraction runs in the
tcgen05 kernel of liblamq_b200.so (bf16 activations, fp32 accumulation); `Statistics` keeps the fp32 accumulators
across chunks (and across ranks: the accumulators are what an all-reduce sums) and `finalize` produces the fp64
H and D.
"""

from __future__ import annotations

import torch

from . import _lib
from ._lib import check, ptr, stream_ptr

CHUNK_TOKENS = 32768  # tokens accumulated on chip before each flush into the fp32 accumulator
MAX_WEIGHT_GROUPS = 4  # distinct token weights handled by gathering (more: the hi/lo split)


def _bf16(x: torch.Tensor) -> torch.Tensor:
    if x.dtype != torch.bfloat16:
        raise TypeError("activations must be bf16 (the model's dtype); got " + str(x.dtype))
    if not x.is_cuda:
        raise RuntimeError("activations must be on a CUDA device")
    x = x.reshape(-1, x.shape[-1])
    if x.stride(-1) != 1 or x.stride(0) % 8 or x.data_ptr() % 16:
        x = x.contiguous()
    return x


class Statistics:
    """fp32 accumulators of one stage's H (and D with a reference stream), fed chunk by chunk."""

    def __init__(self, d: int, cross: bool = False, device=None, chunk_tokens: int = CHUNK_TOKENS):
        dev = torch.device(device or "cuda")
        self.d, self.device, self.chunk_tokens = d, dev, chunk_tokens
        self.accH = torch.zeros(d, d, dtype=torch.float32, device=dev)
        self.accD = torch.zeros(d, d, dtype=torch.float32, device=dev) if cross else None
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self.n_tok = 0

    def _xtx(self, A, B, symmetric, acc, tokens, scale: float = 1.0):
        lib = _lib.load()
        with torch.cuda.device(self.device):
            check(lib.lamq_xtx_accumulate_scaled(ptr(A), A.stride(0), ptr(B), B.stride(0), tokens, self.d,
                                                 1 if symmetric else 0, float(scale), ptr(acc), acc.stride(0),
                                                 self.chunk_tokens, ptr(self.status), stream_ptr(self.device)),
                  "lamq_xtx_accumulate")

    def _gather(self, x, idx):
        out = torch.empty(idx.numel(), self.d, dtype=torch.bfloat16, device=self.device)
        with torch.cuda.device(self.device):
            check(_lib.load().lamq_gather_rows(ptr(x), x.stride(0), ptr(idx), idx.numel(), self.d, ptr(out),
                                               stream_ptr(self.device)), "lamq_gather_rows")
        return out

    def add(self, x: torch.Tensor, w: torch.Tensor | None = None, x_ref: torch.Tensor | None = None,
            weighted=None):
        """One calibration chunk: x (tokens × d bf16, the stream the matrix will see), its token weights w (fp32, or
        None for 1) and, for D, x_ref (the reference stream at the same tokens).

        The main pass takes every token with weight 1 (exact bf16 products); the weighted tokens then add
        Σ (w − 1)·x xᵀ (and Σ (w − 1)·x_ref xᵀ). When they carry at most MAX_WEIGHT_GROUPS distinct weights, the
        tokens of each weight are gathered and added once with scale w − 1 (products still exact); otherwise each
        weighted token enters twice, (w − 1)·x split into a bf16 hi + lo pair. `weighted` may give the groups found
        by the caller as [(device int32 token indices, w), ...]; otherwise they are found here, which reads the
        weights' distinct values back from the device."""
        x = _bf16(x)
        tokens = x.shape[0]
        if x.shape[1] != self.d:
            raise ValueError(f"activations have {x.shape[1]} features, expected {self.d}")
        if (x_ref is not None) != (self.accD is not None):
            raise ValueError("x_ref is required exactly when the statistics include D")
        xr = None if x_ref is None else _bf16(x_ref)
        self._xtx(x, x, True, self.accH, tokens)
        if xr is not None:
            self._xtx(x, xr, False, self.accD, tokens)
        if w is not None:
            w = w.reshape(-1).to(self.device, torch.float32).contiguous()
            if w.numel() != tokens:
                raise ValueError("one weight per token")
            groups = weighted
            if groups is None:
                idx = torch.nonzero(w != 1.0).flatten().to(torch.int32)
                vals = torch.unique(w[idx]).tolist() if idx.numel() else []
                if len(vals) <= MAX_WEIGHT_GROUPS:
                    groups = [(idx[w[idx] == v].contiguous(), v) for v in vals] if len(vals) > 1 else \
                        [(idx, vals[0])] if vals else []
                else:
                    groups = idx
            if isinstance(groups, torch.Tensor):
                self._add_split(x, xr, w, groups)
            else:
                for gidx, v in groups:
                    n = int(gidx.numel())
                    if n == 0:
                        continue
                    xg = self._gather(x, gidx)
                    self._xtx(xg, xg, True, self.accH, n, v - 1.0)
                    if xr is not None:
                        self._xtx(xg, self._gather(xr, gidx), False, self.accD, n, v - 1.0)
        self.n_tok += tokens
        return self

    def _add_split(self, x, xr, w, idx):
        """Σ (w − 1)·x xᵀ for weighted tokens of many distinct weights: (w − 1)·x as a bf16 hi + lo pair."""
        nw = int(idx.numel())
        if nw == 0:
            return
        lib = _lib.load()
        split = torch.empty(2 * nw, self.d, dtype=torch.bfloat16, device=self.device)
        plain = torch.empty_like(split)
        with torch.cuda.device(self.device):
            check(lib.lamq_weighted_split(ptr(x), x.stride(0), ptr(x), x.stride(0), ptr(w), ptr(idx), nw,
                                          self.d, ptr(split), ptr(plain), stream_ptr(self.device)),
                  "lamq_weighted_split")
        # Σ (w−1)·x xᵀ: A = x (plain), B = (w−1)·x (hi and lo rows)
        self._xtx(plain, split, True, self.accH, 2 * nw)
        if xr is not None:
            with torch.cuda.device(self.device):
                check(lib.lamq_weighted_split(ptr(x), x.stride(0), ptr(xr), xr.stride(0), ptr(w), ptr(idx),
                                              nw, self.d, ptr(split), ptr(plain), stream_ptr(self.device)),
                      "lamq_weighted_split")
            # D[j][i] += Σ (w−1)·x[i]·x_ref[j]: A = (w−1)·x (hi and lo), B = x_ref
            self._xtx(split, plain, False, self.accD, 2 * nw)

    def finalize(self, n_tok: int | None = None):
        """(H, D) in fp64: H = acc/n_tok (mirrored from the computed triangle), D = accD/n_tok − H (or None)."""
        n = self.n_tok if n_tok is None else n_tok
        H = torch.empty(self.d, self.d, dtype=torch.float64, device=self.device)
        D = torch.empty_like(H) if self.accD is not None else None
        with torch.cuda.device(self.device):
            check(_lib.load().lamq_hessian_finalize(ptr(self.accH), ptr(self.accD), self.d, self.d, float(n), ptr(H),
                                                    ptr(D), stream_ptr(self.device)), "lamq_hessian_finalize")
        return H, D

    def check_status(self):
        st = int(self.status.item())
        if st:
            _lib.check(st, "Hessian accumulation")


def hessian(x: torch.Tensor, w: torch.Tensor | None = None, x_ref: torch.Tensor | None = None,
            chunk_tokens: int = CHUNK_TOKENS):
    """One-shot H (and D with x_ref) of bf16 activations x (tokens × d) with token weights w."""
    st = Statistics(x.shape[-1], cross=x_ref is not None, device=x.device, chunk_tokens=chunk_tokens)
    st.add(x, w, x_ref)
    return st.finalize()


def main():
    """`python -m lookatmyquant_b200.hessian --tokens 65536 --d 9728`: H and D of random bf16 activations (two passes,
    the second timed with CUDA events); prints the achieved TFLOP/s of each contraction."""
    import argparse
    ap = argparse.ArgumentParser(description=main.__doc__)
    ap.add_argument("--tokens", type=int, default=65536)
    ap.add_argument("--d", type=int, default=9728)
    a = ap.parse_args()
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(a.tokens, a.d, device="cuda", generator=g).to(torch.bfloat16)
    xr = torch.randn(a.tokens, a.d, device="cuda", generator=g).to(torch.bfloat16)
    st = Statistics(a.d, cross=True)
    for rep in range(2):
        for sym, (A, B, acc) in ((True, (x, x, st.accH)), (False, (x, xr, st.accD))):
            s_, e_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s_.record()
            st._xtx(A, B, sym, acc, a.tokens)
            e_.record()
            e_.synchronize()
            ms = s_.elapsed_time(e_)
            fl = 2.0 * a.tokens * a.d * (a.d + 1) / 2 if sym else 2.0 * a.tokens * a.d * a.d
            if rep:
                print(f"d={a.d} tokens={a.tokens} {'H' if sym else 'D'}: {ms:.3f} ms, {fl / ms / 1e9:.1f} TFLOP/s")
    st.check_status()


if __name__ == "__main__":
    main()
