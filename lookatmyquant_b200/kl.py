"""The KL probe's head on B200 (liblamq_b200: lamq_kl_reference, lamq_kl_head).

Reference: compiler.py:176-187 (`measure`): the reference log-probabilities of the held-out windows are taken once,
ref_lp = log_softmax(model(held).logits.float()), and every probe measures
KL = Σ_t w_t·Σ_v exp(ref_lp)·(ref_lp − log_softmax(model(held).logits.float())) / Σ_t w_t.

Here the model's final hidden states (after its final norm) go to the kernel with the LM head; the logits, the
log-softmax and the KL happen in one tcgen05 pass over the vocabulary, and no logits tensor is ever written. The
reference side keeps the distribution (ntok × V fp32, as the reference keeps ref_lp) and three per-position numbers.
"""

from __future__ import annotations

import torch

from . import _lib
from ._lib import check, ptr, stream_ptr


def _bf16_rows(x: torch.Tensor) -> torch.Tensor:
    if x.dtype != torch.bfloat16 or not x.is_cuda:
        raise TypeError("hidden states and the LM head must be bf16 CUDA tensors")
    x = x.reshape(-1, x.shape[-1])
    if x.stride(-1) != 1 or x.stride(0) % 8 or x.data_ptr() % 16:
        x = x.contiguous()
    return x


class KLReference:
    """The reference side of a KL probe: from the unquantized model's final hidden states `h_ref` (positions × d) and
    the LM head `E` (V × d), the reference distribution and per-position statistics. `kl(h, w)` then measures a probe."""

    def __init__(self, h_ref: torch.Tensor, E: torch.Tensor):
        h_ref, E = _bf16_rows(h_ref), _bf16_rows(E)
        if h_ref.shape[1] != E.shape[1]:
            raise ValueError("hidden size and LM head disagree")
        self.E = E
        self.ntok, self.d = h_ref.shape
        self.V = E.shape[0]
        dev = self.device = h_ref.device
        self.ldp = (self.V + 3) // 4 * 4
        self.p = torch.empty(self.ntok, self.ldp, dtype=torch.float32, device=dev)
        self.lse = torch.empty(self.ntok, dtype=torch.float32, device=dev)
        self.A = torch.empty(self.ntok, dtype=torch.float64, device=dev)
        self.P = torch.empty(self.ntok, dtype=torch.float64, device=dev)
        lib = _lib.load()
        self.ws = torch.empty(lib.lamq_kl_workspace_size(self.ntok), dtype=torch.uint8, device=dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        with torch.cuda.device(dev):
            check(lib.lamq_kl_reference(ptr(h_ref), h_ref.stride(0), self.ntok, self.d, ptr(E), E.stride(0), self.V,
                                        ptr(self.p), self.ldp, ptr(self.lse), ptr(self.A), ptr(self.P), ptr(self.ws),
                                        self.ws.numel(), ptr(self.status), stream_ptr(dev)), "lamq_kl_reference")

    def kl(self, h: torch.Tensor, w: torch.Tensor | None = None, per_position: bool = False):
        """The weighted mean KL of the probe's hidden states `h` (same positions) to the reference; with
        `per_position`, also each position's KL (fp32). Synchronizes to read the result."""
        h = _bf16_rows(h)
        if h.shape != (self.ntok, self.d):
            raise ValueError(f"hidden states {tuple(h.shape)}, reference {(self.ntok, self.d)}")
        wv = None if w is None else w.reshape(-1).to(self.device, torch.float32).contiguous()
        if wv is not None and wv.numel() != self.ntok:
            raise ValueError("one weight per position")
        kl_pos = torch.empty(self.ntok, dtype=torch.float32, device=self.device)
        out = torch.empty(3, dtype=torch.float64, device=self.device)
        lib = _lib.load()
        with torch.cuda.device(self.device):
            check(lib.lamq_kl_head(ptr(h), h.stride(0), self.ntok, self.d, ptr(self.E), self.E.stride(0), self.V,
                                   ptr(self.p), self.ldp, ptr(self.lse), ptr(self.A), ptr(self.P), ptr(wv),
                                   ptr(kl_pos), ptr(out), ptr(self.ws), self.ws.numel(), ptr(self.status),
                                   stream_ptr(self.device)), "lamq_kl_head")
        st = int(self.status.item())
        if st:
            _lib.check(st, "KL head")
        value = float(out[0].item())
        return (value, kl_pos) if per_position else value
