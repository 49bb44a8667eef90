"""Trellis codes and block-LDLQ words on B200: the host side of `opgraph.codes` (ShinMegamiBoson/lookatmyquant).

Same names, argument meaning and errors as the reference module, so the reference's callers can bind to it:

    viterbi(X, values, L, k, chunk=None, start=None)            opgraph/codes.py:151-181
    trellis_values(L, k, T=320, seed=0, refine=None, fit=None)  opgraph/codes.py:187-220 (shipped or fitted on the GPU)
    hadamard_factors(n), hadamard(n), rht(n, seed)             opgraph/codes.py:97-132
    is_trellis_path(states, L, k)                               opgraph/codes.py:246-248
    RowTrellisCode(L, k, T=256, width=16, look=8, seed=0)       opgraph/codes.py:386-410
    TrellisCode(L, k, T=320, width=16, seed=0)                  opgraph/codes.py:363-383
    ldlq_words(Ws, H, code, seeds, incoherent=True, in_seed=None, out_rot=True)   opgraph/codes.py:413-462

The compute runs in liblamq_b200.so (sm_100a): the Viterbi decode and the row- and column-trellis sweeps are
hand-written kernels. The words come back as `TrellisWord`s exposing what the reference's callers read from a Net (`matrix()`,
`rate_bits()`, the states and the row scales).
"""

from __future__ import annotations

import math
import os
from pathlib import Path

import numpy as np
import torch

from . import _lib
from ._lib import check, ptr, stream_ptr
from .frame import Environment
from .rotation import Rotation

TABLES = Path(__file__).resolve().parent / "tables"
DEVICE = "cuda"
WIDTH, LOOK, LAZY = 16, 8, 128  # RowTrellisCode's block and look-ahead, sweep's lazy run (codes.py:391, syntax.py:88)


def _dev(device=None) -> torch.device:
    d = torch.device(device or DEVICE)
    if d.type != "cuda":
        raise RuntimeError("lookatmyquant_b200 runs on CUDA devices only (no CPU fallback)")
    return d


# ----------------------------------------------------------------------------- tables


def _table_cache() -> Path:
    return Path(os.environ.get("LAMQ_TABLE_CACHE", Path.home() / ".cache" / "lookatmyquant_b200" / "tables"))


def trellis_values(L: int, k: int, T: int = 320, seed: int = 0, refine: int | None = None, fit: str | None = None
                   ) -> torch.Tensor:
    """The 2^L trellis values for (L, k, T, seed, fit), fp64 on the CPU (codes.py:187-220). The reference's fitted e-means
    tables for T = 256 ship with this package; any other table is fitted once on the GPU (fit_trellis_values) and kept in
    the table cache ($LAMQ_TABLE_CACHE, default ~/.cache/lookatmyquant_b200/tables), as the reference keeps its fits in
    its cache directory."""
    fit = fit or "ema"
    name = f"trellis_L{L}_k{k}_T{T}_s{seed}{'' if fit == 'lloyd' else '_' + fit}.f64"
    if refine is None:
        for path in (TABLES / name, _table_cache() / name):
            if path.exists():
                return torch.from_numpy(np.fromfile(path, dtype="<f8").copy())
    v = fit_trellis_values(L, k, T, seed, refine, fit)
    if refine is None:
        _table_cache().mkdir(parents=True, exist_ok=True)
        tmp = _table_cache() / (name + f".{os.getpid()}.tmp")
        tmp.write_bytes(v.numpy().astype("<f8").tobytes())
        os.replace(tmp, _table_cache() / name)
    return v


def fit_trellis_values(L: int, k: int, T: int, seed: int = 0, refine: int | None = None, fit: str = "ema",
                       device=None) -> torch.Tensor:
    """Fits a table as codes.py:187-220 does: the states' values start as unit-Gaussian quantiles in a random order and
    move to the mean of the Gaussian samples the Viterbi assigns to each state — six Lloyd steps over one set of 4096
    sequences ("lloyd"), or ("ema") 16·384 batches of 256 new sequences whose weight in each state's decaying sum and
    count falls from 0.5 to 0.01 along a cosine. The samples come from torch's CPU generator in the reference's order,
    the Viterbi runs on the GPU (lamq_viterbi, states identical to the reference's), and the per-state sums are kept in
    fp64 on the host with the reference's ops, so the fitted values are the reference's."""
    if fit not in ("lloyd", "ema"):
        raise ValueError(fit)
    dev = _dev(device)
    g = torch.Generator().manual_seed(seed)
    S = 1 << L
    v = torch.special.ndtri((torch.randperm(S, generator=g).double() + 0.5) / S)
    if fit == "lloyd":
        X0 = torch.randn(4096, T, generator=g, dtype=torch.float64)
        batches = ((X0, 1.0) for _ in range(6 if refine is None else refine))
    else:
        steps = 16 * (384 if refine is None else refine)
        batches = ((torch.randn(256, T, generator=g, dtype=torch.float64),
                    0.01 + 0.245 * (1 + math.cos(math.pi * j / max(steps - 1, 1)))) for j in range(steps))
    sums, cnt = torch.zeros(S, dtype=torch.float64), torch.zeros(S, dtype=torch.float64)
    for X, a in batches:
        st = viterbi(X.to(dev), v, L, k).reshape(-1).cpu()
        sums = (1 - a) * sums + a * torch.zeros(S, dtype=torch.float64).index_add_(0, st, X.reshape(-1))
        cnt = (1 - a) * cnt + a * torch.bincount(st, minlength=S).double()
        v = torch.where(cnt > 0, sums / cnt.clamp(min=1e-300), v)
    return v


def stacked_tables(L: int = 12, T: int = 256, device=None) -> torch.Tensor:
    """The four tables k = 1..4 as one (4, 2^L) fp64 device tensor, the layout lamq_ldlq_rowtrellis reads."""
    return torch.stack([trellis_values(L, k, T) for k in (1, 2, 3, 4)]).to(_dev(device))


# ----------------------------------------------------------------------------- the trellis


def viterbi(X: torch.Tensor, values: torch.Tensor, L: int, k: int, chunk: int | None = None,
            start: torch.Tensor | None = None) -> torch.Tensor:
    """The path through a bitshift trellis nearest each row of X in squared error (codes.py:151-181): states
    s_t = (s_{t-1}·2^k + b_t) mod 2^L emitting values[s_t]; with `start`, the state before the first entry is given.
    Costs are fp32 as in the reference, and the states are identical to its. Returns int64 states (rows, T) on X's
    device. `chunk` is accepted for signature compatibility (the kernel needs no row chunking)."""
    dev = _dev(X.device if X.is_cuda else None)
    x = X.to(dev, torch.float32).contiguous()
    if x.dim() != 2:
        raise ValueError("viterbi expects a (rows, T) matrix")
    rows, T = x.shape
    C = values.to(dev, torch.float32).contiguous()
    if C.numel() != 1 << L:
        raise ValueError(f"values must have 2^L = {1 << L} entries")
    st = None if start is None else start.to(dev, torch.int64).contiguous()
    out = torch.empty(rows, T, dtype=torch.int64, device=dev)
    lib = _lib.load()
    ws_bytes = lib.lamq_viterbi_workspace_size(rows, T, L, k)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        check(lib.lamq_viterbi(ptr(x), rows, T, ptr(C), L, k, ptr(st), ptr(out), ptr(ws), ws_bytes,
                               stream_ptr(dev)), "lamq_viterbi")
    return out.to(X.device)


def is_trellis_path(states: torch.Tensor, L: int, k: int) -> bool:
    """codes.py:246-248: every step keeps the previous state's low L − k bits as its high bits."""
    return bool(torch.all((states[..., 1:] >> k) == (states[..., :-1] & ((1 << (L - k)) - 1))))


# ----------------------------------------------------------------------------- Hadamard rotations


def _is_prime(q: int) -> bool:
    return q > 1 and all(q % d for d in range(2, math.isqrt(q) + 1))


def _paley(q: int) -> torch.Tensor:
    """Paley's first construction of order q + 1 for a prime q ≡ 3 (mod 4) (codes.py:87-94)."""
    sq = {(x * x) % q for x in range(1, q)}
    chi = torch.tensor([0.0] + [1.0 if a in sq else -1.0 for a in range(1, q)], dtype=torch.float64)
    Q = chi[(torch.arange(q)[None, :] - torch.arange(q)[:, None]) % q]
    S = torch.zeros(q + 1, q + 1, dtype=torch.float64)
    S[0, 1:], S[1:, 0], S[1:, 1:] = 1, -1, Q
    return S + torch.eye(q + 1, dtype=torch.float64)


def _sylvester(a: int) -> torch.Tensor:
    H = torch.ones(1, 1, dtype=torch.float64)
    while H.shape[0] < 2 ** a:
        H = torch.cat([torch.cat([H, H], 1), torch.cat([H, -H], 1)], 0)
    return H


def hadamard_factors(n: int) -> tuple[torch.Tensor, torch.Tensor]:
    """A and B with hadamard(n) = (A ⊗ B)/√n (codes.py:104-119)."""
    for a in range(int(math.log2(n)), -1, -1):
        if n % 2 ** a:
            continue
        p = n // 2 ** a
        if p in (1, 2) or (_is_prime(p - 1) and (p - 1) % 4 == 3):
            if p == 1 and a > 1:
                return _sylvester(a // 2), _sylvester(a - a // 2)
            P = (torch.tensor([[1.0, 1.0], [1.0, -1.0]], dtype=torch.float64) if p == 2
                 else torch.ones(1, 1, dtype=torch.float64) if p == 1 else _paley(p - 1))
            return _sylvester(a), P
    raise ValueError(f"no Hadamard construction here for order {n}")


def hadamard(n: int) -> torch.Tensor:
    A, B = hadamard_factors(n)
    return torch.kron(A, B) / math.sqrt(n)


def rht_signs(n: int, seed: int) -> torch.Tensor:
    """The random signs of rht(n, seed) (codes.py:131), from torch's CPU generator as the reference draws them."""
    u = torch.rand(n, generator=torch.Generator().manual_seed(int(seed)), dtype=torch.float64)
    return torch.where(u < 0.5, -1.0, 1.0).to(torch.float64)


def rht(n: int, seed: int) -> torch.Tensor:
    """A randomized Hadamard transform hadamard(n)·diag(s) (codes.py:129-132), fp64 on the CPU."""
    return hadamard(n) * rht_signs(n, seed)[None, :]


# ----------------------------------------------------------------------------- codes


class RowTrellisCode:
    """Each row as one trellis path along its columns, from state 0 (codes.py:386-410). Block LDLQ settles `width`
    columns at a time; each block's Viterbi also looks `look` columns ahead."""

    def __init__(self, L: int, k: int, T: int = 256, width: int = 16, look: int = 8, seed: int = 0, values=None):
        self.L, self.k, self.T, self.width, self.look, self.seed = L, k, T, width, look, seed
        self.values = trellis_values(L, k, T, seed) if values is None else torch.as_tensor(values).double().cpu()
        self.state = None

    def step(self, j, X, ahead):
        """Column j onward, `width` columns: the block's settled values, continuing each row's path (codes.py:397-404)."""
        if j == 0:
            self.state = torch.zeros(len(X), dtype=torch.long, device=X.device)
        w = X.shape[1]
        path = viterbi(torch.cat([X, ahead], 1), self.values, self.L, self.k, start=self.state)[:, :w]
        self.state = path[:, -1]
        return self.values.to(X.device, X.dtype)[path]


class TrellisCode:
    """Sequences of T consecutive outputs (one column) onto trellis paths (codes.py:363-383)."""

    def __init__(self, L: int, k: int, T: int = 320, width: int = 16, seed: int = 0, values=None):
        self.L, self.k, self.T, self.width, self.seed = L, k, T, width, seed
        self.values = trellis_values(L, k, T, seed) if values is None else torch.as_tensor(values).double().cpu()

    def _seqs(self, X):
        o, w = X.shape
        return X.reshape(o // self.T, self.T, w).permute(0, 2, 1).reshape(-1, self.T)

    def project(self, X):
        o, w = X.shape
        Q = self.values.to(X.device, X.dtype)[viterbi(self._seqs(X), self.values, self.L, self.k)]
        return Q.reshape(o // self.T, w, self.T).permute(0, 2, 1).reshape(o, w)


class _Domain:
    """What a Net core records of its code (frame.py's domain): the value table and whether sequences start at 0."""

    def __init__(self, levels, fixed_start):
        self.levels, self.fixed_start = levels, fixed_start


class _Core:
    """A Net core's tensor (`.data`) and, for the code core, its domain."""

    def __init__(self, data, domain=None):
        self.data, self.domain = data, domain


class TrellisWord:
    """One matrix's trellis word: W ≈ R_outᵀ·diag(S)·V[states]·R_in. The fields are device tensors:
    `states` (rows × n int16), `scales` S (rows fp64), `settled` V[states] (fp64, units of S); the rotations are
    `Rotation`s (None: no rotation on that side)."""

    def __init__(self, states, scales, settled, values, L, k, in_seed, R_in, R_out=None, fixed_start=True, T=None):
        self.states, self.scales, self.settled, self.values = states, scales, settled, values
        self.L, self.k, self.in_seed, self.R_in, self.R_out = L, k, in_seed, R_in, R_out
        self.fixed_start, self.T = fixed_start, T

    def matrix(self, device=None, dtype=torch.float64) -> torch.Tensor:
        """The dequantized matrix (reference Net.matrix, frame.py:112-134): diag(S)·V[states]·R_in, then R_outᵀ·."""
        W = self.settled * self.scales[:, None]
        if self.R_in is not None:
            W = self.R_in.rows_t(W)
        if self.R_out is not None:
            W = self.R_out.rows_t(W.T.contiguous()).T.contiguous()
        return W.to(device=device or W.device, dtype=dtype)

    @property
    def cores(self) -> dict:
        """The reference Net's cores that its callers read (quantize.py:513-527, :1541-1552): "W" (the settled table
        values, with the code's `domain.levels` and `domain.fixed_start`), "W.S" (the row scales), and "I[u]" (the
        output signs) when the word has an output rotation."""
        levels = self.values.double().cpu() if hasattr(self.values, "double") else self.values
        out = {"W": _Core(self.settled, _Domain(levels, self.fixed_start)), "W.S": _Core(self.scales[:, None])}
        if self.R_out is not None:
            out["I[u]"] = _Core(getattr(self.R_out, "signs", None))
        return out

    def rate_bits(self) -> float:
        """Stored bits (frame.py:137-147): k per entry, plus L − k per sequence without a fixed start, 16 per row
        scale, one sign per input (and per output with an output rotation)."""
        m, n = self.states.shape
        bits = float(m * n * self.k) + 16.0 * m + (n if self.R_in is not None else 0) + (m if self.R_out is not None else 0)
        if not self.fixed_start:
            bits += (m * n / self.T) * (self.L - self.k)
        return bits


# ----------------------------------------------------------------------------- words


def _row_trellis_sweep(X, S, env, code, row_bits=None, settled_out=True):
    """The fused sweep kernel: X (rows × n fp64, device) is settled in place; returns (before, states, settled)."""
    dev = X.device
    rows, n = X.shape
    T = X.contiguous().clone()
    states = torch.empty(rows, n, dtype=torch.int16, device=dev)
    settled = torch.empty(rows, n, dtype=torch.float64, device=dev) if settled_out else None
    tables = stacked_tables(code.L, code.T, dev) if code.L == 12 else None
    if tables is None:
        raise ValueError("the fused sweep supports L = 12")
    if row_bits is None:
        tables[code.k - 1] = code.values.to(dev)
    dead = env.dead.to(dev, torch.uint8) if bool(env.dead.any()) else None
    ws = torch.empty(_lib.load().lamq_ldlq_rowtrellis_workspace_size(rows, n), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        check(_lib.load().lamq_ldlq_rowtrellis(
            ptr(T), n, rows, n, ptr(env.U), env.U.stride(0), ptr(dead), ptr(S.contiguous()), ptr(tables),
            ptr(row_bits), code.k, code.L, code.width, code.look, LAZY, ptr(states), ptr(settled),
            ptr(ws), ws.numel(), stream_ptr(dev)), "lamq_ldlq_rowtrellis")
    return T, states, settled


def _col_trellis_sweep(X, S, env, code, settled_out=True):
    """lamq_ldlq_coltrellis: the column-trellis sweep of X (rows × n fp64, device); returns (before, states, settled)."""
    dev = X.device
    rows, n = X.shape
    if rows % code.T:
        raise ValueError(f"{rows} rows are not a whole number of runs of {code.T}")
    T = X.contiguous().clone()
    states = torch.empty(rows, n, dtype=torch.int16, device=dev)
    settled = torch.empty(rows, n, dtype=torch.float64, device=dev) if settled_out else None
    table = code.values.to(dev, torch.float64).contiguous()
    dead = env.dead.to(dev, torch.uint8) if bool(env.dead.any()) else None
    lib = _lib.load()
    ws = torch.empty(lib.lamq_ldlq_coltrellis_workspace_size(rows, n, code.T, code.L, code.k, code.width, LAZY),
                     dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        check(lib.lamq_ldlq_coltrellis(ptr(T), n, rows, n, ptr(env.U), env.U.stride(0), ptr(dead), ptr(S.contiguous()),
                                       ptr(table), code.k, code.L, code.T, code.width, LAZY, ptr(states), ptr(settled),
                                       ptr(ws), ws.numel(), stream_ptr(dev)), "lamq_ldlq_coltrellis")
    return T, states, settled


def generic_trellis_sweep(X, S, env, code):
    """The sweep of ldlq_words (codes.py:442-450) for trellises the fused kernels do not take (L < 12): the generic
    block sweep (syntax.sweep, the reference's order, the run product on the fp64 tensor cores) with the code's
    projection — RowTrellisCode.step (each row's path continued from its last state over the block and `look` columns
    ahead) or TrellisCode.project (runs of T rows down each column) — through lamq_viterbi's kernel for fewer states.
    X (rows × n fp64, device). Returns (states int16, settled values in units of S, fp64)."""
    from .syntax import sweep
    rows, n = X.shape
    dev = X.device
    settled = torch.empty_like(X)
    states = torch.empty(rows, n, dtype=torch.int16, device=dev)
    values = code.values.to(dev, torch.float64)
    last = [torch.zeros(rows, dtype=torch.long, device=dev)]

    def project(j, x, T):
        xs = x[:, None] if code.width == 1 else x
        w = xs.shape[1]
        if isinstance(code, RowTrellisCode):
            win = torch.cat([xs / S[:, None], T[:, j + w:j + w + code.look] / S[:, None]], 1)
            path = viterbi(win, code.values, code.L, code.k, start=last[0])[:, :w]
            last[0] = path[:, -1]
        else:
            o = xs.shape[0]
            seqs = (xs / S[:, None]).reshape(o // code.T, code.T, w).permute(0, 2, 1).reshape(-1, code.T)
            path = viterbi(seqs, code.values, code.L, code.k)
            path = path.reshape(o // code.T, w, code.T).permute(0, 2, 1).reshape(o, w)
        q = values[path]
        settled[:, j:j + w] = q
        states[:, j:j + w] = path.to(torch.int16)
        q = q * S[:, None]
        return q[:, 0] if code.width == 1 else q

    sweep(X, env, project, width=code.width)
    return states, settled


def _gaussian_centroids(bounds: torch.Tensor) -> torch.Tensor:
    """The mean of a unit Gaussian on each cell [bounds[j], bounds[j+1]] (nested.py:44-48)."""
    phi = lambda x: torch.exp(-0.5 * x * x) / math.sqrt(2 * math.pi)
    Phi = lambda x: 0.5 * (1 + torch.erf(x / math.sqrt(2)))
    a, b = bounds[:-1], bounds[1:]
    pa = torch.where(torch.isinf(a), torch.zeros_like(a), phi(a))
    pb = torch.where(torch.isinf(b), torch.zeros_like(b), phi(b))
    return (pa - pb) / (Phi(b) - Phi(a))


def lloyd_max_levels(n: int, iters: int = 500) -> torch.Tensor:
    """The best n levels for a unit Gaussian (nested.py:75-82): fp64 on the CPU."""
    lv = _gaussian_centroids(torch.special.ndtri(torch.arange(n + 1, dtype=torch.float64) / n) * math.sqrt(3))
    for _ in range(iters):
        mid = (lv[1:] + lv[:-1]) / 2
        bounds = torch.cat([torch.tensor([-math.inf], dtype=lv.dtype), mid, torch.tensor([math.inf], dtype=lv.dtype)])
        lv = _gaussian_centroids(bounds)
    return lv


def synthetic_codebook(bits: int, seed: int = 0) -> tuple[int, torch.Tensor]:
    """BASELINE config 3's codebook for a width: a Lloyd-Max fit to N(0, 1) with 2^(bits+4) entries rounded to fp16,
    placed in state order as trellis_values orders its quantiles (codes.py:202-204: state s takes the level of rank
    randperm(2^L)[s], torch's CPU generator seeded `seed`). Returns (L, values fp64)."""
    L = bits + 4
    S = 1 << L
    levels = lloyd_max_levels(S).to(torch.float16).double()
    perm = torch.randperm(S, generator=torch.Generator().manual_seed(seed))
    return L, levels[perm]


def _round_to_nearest(X, S, code):
    """The code applied directly, without H (codes.py:460-461 with `settled` None): each row from state 0 (row trellis,
    codes.py:406-409) or each run of T outputs down a column (column trellis, codes.py:371-378)."""
    xs = X / S[:, None]
    if isinstance(code, RowTrellisCode):
        st = viterbi(xs, code.values, code.L, code.k, start=torch.zeros(len(xs), dtype=torch.long, device=xs.device))
    else:
        o, w = xs.shape
        st = viterbi(code._seqs(xs), code.values, code.L, code.k)
        st = st.reshape(o // code.T, w, code.T).permute(0, 2, 1).reshape(o, w)
    return st.to(torch.int16), code.values.to(X.device, torch.float64)[st]


def ldlq_words(Ws: list[torch.Tensor], H: torch.Tensor | None, code, seeds: list[int], incoherent: bool = True,
               in_seed: int | None = None, out_rot: bool = True, device=None) -> list[TrellisWord]:
    """(Gauge: incoherence →) Split(scale, per row, by RMS) → (block LDLQ sweep →) the trellis code, for matrices that
    read the same input (codes.py:413-462), on the GPU in fp64. Matrices are swept together (rows do not interact
    under Refit). Returns one TrellisWord per matrix."""
    dev = _dev(device)
    Ws = [W.to(dev, torch.float64) for W in Ws]
    n = Ws[0].shape[1]
    R_in = Rotation(n, seeds[0] + 1 if in_seed is None else in_seed, dev) if incoherent else None
    Xs, R_outs = [], []
    for W, s in zip(Ws, seeds):
        X = R_in.rows(W) if incoherent else W
        if incoherent and out_rot:
            R_out = Rotation(W.shape[0], s, dev)
            X = R_out.rows(X.T.contiguous()).T.contiguous()  # R_out·(W·R_inᵀ)
            R_outs.append(R_out)
        else:
            R_outs.append(None)
        Xs.append(X)
    X = torch.cat(Xs) if len(Xs) > 1 else Xs[0]
    S = X.pow(2).mean(1).sqrt().clamp(min=1e-12)
    if not isinstance(code, (RowTrellisCode, TrellisCode)):
        raise TypeError(f"unsupported code {type(code).__name__}")
    if H is None:
        states, settled = _round_to_nearest(X, S, code)
    else:
        Hd = H.to(dev, torch.float64)
        env = Environment(R_in.conj(Hd) if incoherent else Hd)
        if code.L != 12:  # fewer states than the fused kernels take: the generic sweep with the small Viterbi
            states, settled = generic_trellis_sweep(X, S, env, code)
        else:
            sweep = _row_trellis_sweep if isinstance(code, RowTrellisCode) else _col_trellis_sweep
            _, states, settled = sweep(X, S, env, code)
        env.check()
    fixed, T = (True, None) if isinstance(code, RowTrellisCode) else (False, code.T)
    out, r0 = [], 0
    for W, R_out in zip(Ws, R_outs):
        r1 = r0 + W.shape[0]
        out.append(TrellisWord(states[r0:r1], S[r0:r1], settled[r0:r1], code.values, code.L, code.k,
                               in_seed, R_in, R_out, fixed, T))
        r0 = r1
    return out


def main():
    """`python -m lookatmyquant_b200.codes fit --k 2 3 4 --T 320 --out DIR`: fits tables on the GPU (fit_trellis_values)
    and writes them as raw little-endian fp64 files named as the package's tables, with their SHA-256 sums."""
    import argparse
    import hashlib
    import time
    ap = argparse.ArgumentParser(description=main.__doc__)
    ap.add_argument("command", choices=["fit", "sweep"])
    ap.add_argument("--rows", type=int, default=1024)
    ap.add_argument("--n", type=int, default=2560)
    ap.add_argument("--L", type=int, default=12)
    ap.add_argument("--k", type=int, nargs="+", default=[2, 3, 4])
    ap.add_argument("--T", type=int, default=320)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--fit", default="ema", choices=["ema", "lloyd"])
    ap.add_argument("--out", type=Path)
    a = ap.parse_args()
    if a.command == "sweep":
        _sweep_cli(a.rows, a.n, a.k[0])
        return
    a.out.mkdir(parents=True, exist_ok=True)
    for k in a.k:
        t0 = time.time()
        v = fit_trellis_values(a.L, k, a.T, a.seed, None, a.fit)
        name = f"trellis_L{a.L}_k{k}_T{a.T}_s{a.seed}{'' if a.fit == 'lloyd' else '_' + a.fit}.f64"
        raw = v.numpy().astype("<f8").tobytes()
        (a.out / name).write_bytes(raw)
        shipped = TABLES / name
        note = ""
        if shipped.exists():
            ref = np.fromfile(shipped, dtype="<f8")
            note = f" max |fit - shipped| {np.abs(ref - v.numpy()).max():.3e}"
        print(f"{hashlib.sha256(raw).hexdigest()}  {name}  ({time.time() - t0:.1f} s){note}", flush=True)


def _sweep_cli(rows: int, n: int, k: int):
    """One row-trellis sweep of a random rows × n word at width k under a random H (two launches, the second timed)."""
    g = torch.Generator(device="cuda").manual_seed(0)
    A = torch.randn(2 * n, n, device="cuda", dtype=torch.float64, generator=g)
    A = A * torch.exp(torch.randn(n, device="cuda", dtype=torch.float64, generator=g))
    env = Environment(A.T @ A / (2 * n))
    X = 0.02 * torch.randn(rows, n, device="cuda", dtype=torch.float64, generator=g)
    S = X.pow(2).mean(1).sqrt()
    code = RowTrellisCode(12, k)
    rb = torch.full((rows,), k, dtype=torch.uint8, device="cuda")
    for rep in range(2):
        s_, e_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s_.record()
        _row_trellis_sweep(X, S, env, code, row_bits=rb)
        e_.record()
        e_.synchronize()
    print(f"sweep {rows} x {n}, k = {k}: {s_.elapsed_time(e_):.3f} ms")


if __name__ == "__main__":
    main()
