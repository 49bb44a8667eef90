"""The per-matrix entry of the reference's build (`quantize.word`) for the programs on the B200 path.

Reference: quantize.py:96 (program names), :276-285 (`parse`), :288-298 (`Dense`), :332-347 (`word`), :1316-1328
(`best_word`: the seed with the least H-weighted error). `word(program,
W, H, seed, trellis, in_seed, out_rot, G)` returns a Net-like object with `matrix(dtype)`, `rate_bits()` and — for
the trellis programs — `cores["W"]` / `cores["W.S"]`, which quantize.py reads to save codes (:513-527, :1541-1552).

The trellis programs (`tr{b}`, and `tr{b}x`, whose cross term only changes the target the caller passes) run the
fused sweep (codes.ldlq_words); `fp16` keeps the checkpoint's bf16 values. The other families the reference offers
(rtn, gptq, gptaq, higgs, lm, ter) are not part of this hot path and raise NotImplementedError.
"""

from __future__ import annotations

import re

import torch

from . import codes
from .frame import proxy_loss

PROGRAM = re.compile(r"orig|(rtn|gptq|gptaq|lm|tr|higgs|ter)(\d)(x?)")


def parse(program: str):
    """(family, bits, cross-term target) of a program name, as quantize.parse reads it."""
    if program == "fp16":
        return "fp", 16, False
    if program in ("mean", "prng", "zero"):
        return program, 0, False
    m = PROGRAM.fullmatch(program)
    if not m or not m.group(1) or (m.group(1) in ("gptaq", "rtn", "gptq", "higgs") and m.group(3)):
        raise ValueError(f"unknown program {program}")
    return m.group(1), int(m.group(2)), m.group(1) == "gptaq" or m.group(3) == "x"


class Dense:
    """A matrix kept as its dense reconstruction, with the bits its format stores."""

    def __init__(self, W: torch.Tensor, bits: float):
        self.W, self.bits = W, bits

    def matrix(self, dtype=torch.float64) -> torch.Tensor:
        return self.W.to(dtype)

    def rate_bits(self) -> float:
        return self.bits


def word(program: str, W: torch.Tensor, H: torch.Tensor, seed: int, trellis: dict, in_seed: int | None = None,
         out_rot: bool = True, G: torch.Tensor | None = None):
    """One matrix's quantized word for its target W and input statistics H: `trellis[b]` is the code of width b
    (codes.RowTrellisCode or codes.TrellisCode)."""
    fam, b, _ = parse(program)
    if fam == "fp":
        return Dense(W.to(torch.bfloat16).double(), 16 * W.numel())
    if fam == "tr":
        if G is not None:
            raise NotImplementedError("output-weighted (G) trellis words are not on the B200 path")
        return codes.ldlq_words([W], H, trellis[b], [seed], in_seed=in_seed, out_rot=out_rot)[0]
    raise NotImplementedError(f"program family {fam!r} is outside the B200 hot path (trellis codes)")


SEED_STEP = 7919  # best_word's seed stride between candidates (quantize.py:1323)


def best_word(program: str, target: torch.Tensor, H: torch.Tensor | None, seed: int, trellis: dict, seeds: int = 1,
              in_seed: int | None = None, out_rot: bool = True, G: torch.Tensor | None = None):
    """quantize.py:1316-1328: the program's word; with `seeds` > 1 (the reference's --seeds), the randomized Hadamard
    seed — an exact choice — with the least H-weighted error (E @ H * E).sum(), E = word − target, the first on ties.
    As in the reference, the candidates are `word(program, target, H, seed + 7919·t, trellis)` with the default input
    seed and output rotation. The errors are computed on the device (lamq_proxy_loss) and compared there; the host
    reads one index at the end. Returns (word, errors) with errors None for a single word."""
    fam = parse(program)[0]
    if seeds <= 1 or H is None or fam not in ("tr", "lm"):
        return word(program, target, H, seed, trellis, in_seed, out_rot, G), None
    if fam != "tr":
        raise NotImplementedError(f"program family {fam!r} is outside the B200 hot path (trellis codes)")
    dev = H.device if H.is_cuda else torch.device(codes.DEVICE)
    Hd = H.to(dev, torch.float64)
    tgt = target.to(dev, torch.float64)
    nets, errs = [], []
    for t in range(seeds):
        net = word(program, target, H, seed + SEED_STEP * t, trellis)
        nets.append(net)
        errs.append(proxy_loss(net.matrix(device=dev), tgt, Hd))
    errs = torch.stack(errs)
    return nets[int(torch.argmin(errs).item())], errs
