"""Embedding tables by frequency buckets on B200: the host side of quantize.py's `embedding_buckets`,
`frequency_order`, `embed_word` and `quantize_embedding` (ShinMegamiBoson/lookatmyquant, quantize.py:350-365,
:395-465) for the trellis family and the bucket programs without a code.

A bucket of embedding rows is rotated over the hidden dimension only (each row stays its own, so a lookup decodes one
row), split into a 16-bit RMS scale per row, and coded with a column trellis over runs of 256 rows (TrellisCode with
T = 256: down each hidden column, 256 consecutive rows form one free-start path) — under block LDLQ with the table's
input statistics H, or by plain Viterbi rounding when H is None or the identity (a lookup table). Rows are padded with
zero rows to whole runs of 256 and dropped after. The compute runs in liblamq_b200.so: the rotation through the
Hadamard factors (lamq_rht_rows), the environment (lamq_env_factor), the column-trellis sweep (lamq_ldlq_coltrellis)
or the Viterbi (lamq_viterbi). `lm`/`ter` scalar-code buckets and sliced (per-layer-input) tables are not on this
path and raise NotImplementedError.
"""

from __future__ import annotations

import torch

from . import codes
from .quantize import Dense, parse
from .rotation import Rotation

EMBED_T = 256  # embedding rows per trellis run (quantize.py:99)


def embedding_buckets(V: int, first: int = 256) -> list:
    """Sizes of the buckets of a V-row table ranked by frequency (quantize.py:350-358): first, first, then doubling,
    the last bucket the rest."""
    sizes, s = [first], first
    while sum(sizes) + s < V:
        sizes.append(s)
        s *= 2
    return sizes + [V - sum(sizes)]


def frequency_order(ids: torch.Tensor, V: int) -> torch.Tensor:
    """Token ids by count in `ids`, most frequent first, ties by id (quantize.py:361-364)."""
    counts = torch.bincount(ids.reshape(-1).cpu(), minlength=V)[:V]
    return torch.sort(-counts, stable=True).indices


def embed_word(W: torch.Tensor, H: torch.Tensor | None, program: str, seed: int, center: bool = False,
               device=None):
    """One bucket of embedding rows (quantize.py:395-446): a Dense word (the dequantized rows, fp64 on the device, and
    the bits its format stores). Families: tr<b> (column trellis over runs of 256 rows, L = 12, the package's T = 256
    tables), fp16, mean, zero, prng; `center` stores the bucket's mean row apart (16 bits a value)."""
    dev = codes._dev(device)
    fam, b, _ = parse(program)
    W = W.to(dev)
    if center and fam not in ("fp", "mean", "prng", "zero"):
        m = W.double().mean(0, keepdim=True)
        q = embed_word(W.double() - m, H, program, seed, device=dev)
        return Dense(q.matrix() + m, q.rate_bits() + 16 * W.shape[1])
    if fam == "fp":
        return Dense(W.to(torch.bfloat16).double(), 16 * W.numel())
    if fam == "mean":
        return Dense(W.double().mean(0, keepdim=True).expand_as(W).clone(), 16 * W.shape[1])
    if fam == "zero":
        return Dense(torch.zeros_like(W, dtype=torch.float64), 0)
    if fam == "prng":  # what is stored: the mean row and each column's spread; the noise from torch's CPU generator
        m = W.double().mean(0, keepdim=True)
        noise = torch.randn(W.shape, generator=torch.Generator().manual_seed(seed), dtype=torch.float64).to(dev)
        return Dense(m + noise * (W.double() - m).std(0, keepdim=True), 32 * W.shape[1])
    if fam != "tr":
        raise NotImplementedError(f"embedding program family {fam!r} is outside the B200 hot path (trellis codes)")
    n = W.shape[1]
    lookup = H is None or bool(torch.equal(H.cpu().double(), torch.eye(len(H), dtype=torch.float64)))
    R = Rotation(n, seed, dev)
    rows = W.shape[0]
    pad = (-rows) % EMBED_T
    Wp = torch.cat([W.double(), torch.zeros(pad, n, dtype=torch.float64, device=dev)]) if pad else W.double()
    # the reference rotates in fp32 (a wide table is a large product); the values are rounded to fp32 as it does
    Wr = R.rows(Wp.float().double()).float().double()
    Hr = None if lookup else R.conj(H.to(dev, torch.float64))
    code = codes.TrellisCode(12, b, T=EMBED_T)
    net = codes.ldlq_words([Wr], Hr, code, [seed], incoherent=False, device=dev)[0]
    Q = net.matrix(dtype=torch.float64)[:rows]
    out = R.rows_t(Q.float().double()).float().double()
    return Dense(out, net.rate_bits() * rows / (rows + pad))


@torch.no_grad()
def quantize_embedding(E: torch.Tensor, spec: dict, H: torch.Tensor | None, order: torch.Tensor, seed0: int = 7000,
                       center: bool = False, seed_shift: int = 0):
    """One table, bucket by bucket as the plan says (quantize.py:449-465): spec = {"sizes": [...], "programs": [...]},
    `order` the rows by frequency. E is written in place with each bucket's dequantized rows; returns (bits, weights)."""
    bits, lo = 0.0, 0
    for k, (size, p) in enumerate(zip(spec["sizes"], spec["programs"])):
        rows = order[lo:lo + size].to(E.device)
        net = embed_word(E.data[rows].double(), H, p, seed0 + k + seed_shift, center=center, device=E.device)
        E.data[rows] = net.matrix(dtype=torch.float64).to(E.dtype).to(E.device)
        bits += net.rate_bits()
        lo += size
    return bits, E.numel()
