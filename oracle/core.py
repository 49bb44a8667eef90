"""TEST INFRASTRUCTURE ONLY — CPU restatement of the reference's quantization-build hot path (the parity oracle).

Only `tests/`, `__graft_entry__.smoke()` and `bench.py`'s CPU-baseline leg use this module. Citations are
`file:line` in ShinMegamiBoson/lookatmyquant.
"""

from __future__ import annotations

import ctypes
import math
import os
import subprocess
import threading
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB = None
_LOCK = threading.Lock()


def _lib():
    """The C restatement of `viterbi` (oracle/viterbi.c), built on first use with oracle/Makefile."""
    global _LIB
    with _LOCK:
        if _LIB is None:
            so = _HERE / "_build" / "liboracle.so"
            if not so.exists() or so.stat().st_mtime < (_HERE / "viterbi.c").stat().st_mtime:
                subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)
            lib = ctypes.CDLL(str(so))
            lib.oracle_viterbi.restype = ctypes.c_int
            lib.oracle_viterbi.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                                           ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
            _LIB = lib
    return _LIB


def set_threads(n: int | None):
    """Threads the C Viterbi may use (OpenMP); None leaves the runtime's default."""
    if n is not None:
        os.environ["OMP_NUM_THREADS"] = str(int(n))


# ----------------------------------------------------------------------------- the trellis (codes.py:151-181)


def viterbi(X, values, L: int, k: int, start=None) -> np.ndarray:
    """`opgraph.codes.viterbi` (codes.py:151-181): the trellis path nearest each row of X in squared error, fp32 costs.
    X (rows, T) is rounded to fp32 as the reference's `.to(torch.float32)` does (codes.py:162); values to fp32
    (codes.py:159). Returns int64 states (rows, T)."""
    X = np.ascontiguousarray(np.asarray(X, dtype=np.float64).astype(np.float32))
    C = np.ascontiguousarray(np.asarray(values, dtype=np.float64).astype(np.float32))
    assert C.shape == (1 << L,), C.shape
    rows, T = X.shape
    out = np.empty((rows, T), dtype=np.int64)
    st = None
    if start is not None:
        st = np.ascontiguousarray(np.asarray(start, dtype=np.int64).reshape(rows))
    if rows and T:
        _lib().oracle_viterbi(X.ctypes.data, rows, T, C.ctypes.data, L, k, None if st is None else st.ctypes.data,
                              out.ctypes.data)
    return out


def is_trellis_path(states, L: int, k: int) -> bool:
    """codes.py:246-248: every step keeps the previous state's low L − k bits as its high bits."""
    s = np.asarray(states, dtype=np.int64)
    return bool(np.all((s[..., 1:] >> k) == (s[..., :-1] & ((1 << (L - k)) - 1))))


def viterbi_bruteforce(x, values, L: int, k: int) -> float:
    """The minimum squared error over every path (the check of tests/test_codes.py:101-117); tiny L and T only."""
    import itertools
    best = math.inf
    for s0 in range(1 << L):
        for bits in itertools.product(range(1 << k), repeat=len(x) - 1):
            s, cost = s0, (x[0] - values[s0]) ** 2
            for t, b in enumerate(bits, 1):
                s = ((s << k) | b) & ((1 << L) - 1)
                cost += (x[t] - values[s]) ** 2
            best = min(best, cost)
    return best


# ----------------------------------------------------------------------------- Hadamard rotations (codes.py:83-132)


def _is_prime(q: int) -> bool:
    return q > 1 and all(q % d for d in range(2, math.isqrt(q) + 1))


def paley(q: int) -> np.ndarray:
    """Paley's first construction of order q + 1 (codes.py:87-94): [[1, 1…1], [−1, Q + I]] with Q the Jacobsthal
    matrix Q[i, j] = χ((j − i) mod q), χ the quadratic character."""
    sq = {(x * x) % q for x in range(1, q)}
    chi = np.array([0.0] + [1.0 if a in sq else -1.0 for a in range(1, q)])
    idx = (np.arange(q)[None, :] - np.arange(q)[:, None]) % q
    S = np.zeros((q + 1, q + 1))
    S[0, 1:] = 1
    S[1:, 0] = -1
    S[1:, 1:] = chi[idx]
    return S + np.eye(q + 1)


def sylvester(a: int) -> np.ndarray:
    H = np.ones((1, 1))
    while H.shape[0] < 2 ** a:
        H = np.block([[H, H], [H, -H]])
    return H


def hadamard_factors(n: int):
    """codes.py:104-119: (A, B) with hadamard(n) = (A ⊗ B)/√n; the largest power of two first, Paley for the rest,
    a pure power of two split in the middle."""
    for a in range(int(math.log2(n)), -1, -1):
        if n % 2 ** a:
            continue
        p = n // 2 ** a
        if p in (1, 2) or (_is_prime(p - 1) and (p - 1) % 4 == 3):
            if p == 1 and a > 1:
                return sylvester(a // 2), sylvester(a - a // 2)
            P = np.array([[1.0, 1.0], [1.0, -1.0]]) if p == 2 else np.ones((1, 1)) if p == 1 else paley(p - 1)
            return sylvester(a), P
    raise ValueError(f"no Hadamard construction here for order {n}")


def hadamard(n: int) -> np.ndarray:
    A, B = hadamard_factors(n)
    return np.kron(A, B) / math.sqrt(n)


def rht_signs(n: int, seed: int) -> np.ndarray:
    """codes.py:131: s = −1 where torch.rand(n, seed, float64) < 0.5, else +1 (torch's CPU generator defines them)."""
    import torch
    u = torch.rand(n, generator=torch.Generator().manual_seed(int(seed)), dtype=torch.float64).numpy()
    return np.where(u < 0.5, -1.0, 1.0)


def rht(n: int, seed: int) -> np.ndarray:
    """codes.py:129-132: hadamard(n) · diag(s)."""
    return hadamard(n) * rht_signs(n, seed)[None, :]


# ----------------------------------------------------------------------------- the environment (frame.py:515-522)


def environment(H, damp: float = 0.01):
    """frame.py:515-522: dead inputs (zero diagonal) get a unit diagonal, H += damp·mean(diag H)·I, and
    U = chol(cholesky_inverse(chol(H)))ᵀ, the upper Cholesky factor of H⁻¹. Returns (U, dead, H_damped)."""
    import scipy.linalg as sl
    H = np.array(H, dtype=np.float64, copy=True)
    dead = np.diag(H) == 0
    idx = np.nonzero(dead)[0]
    H[idx, idx] = 1
    H += damp * np.mean(np.diag(H)) * np.eye(len(H))
    Lc = np.linalg.cholesky(H)
    Li = sl.solve_triangular(Lc, np.eye(len(H)), lower=True)
    Hinv = Li.T @ Li
    U = np.linalg.cholesky(Hinv).T
    return U, dead, H


# ----------------------------------------------------------------------------- the block-LDLQ sweep (syntax.py:86-124)


def row_trellis_sweep(X, S, U, dead, values, L: int, k: int, width: int = 16, look: int = 8, lazy: int = 128,
                      on_viterbi=None):
    """`sweep` (syntax.py:86-124) with `RowTrellisCode.step` (codes.py:397-404) as the projection of `ldlq_words`
    (codes.py:442-450). Each block of `width` columns is settled by a Viterbi over the block plus `look` columns ahead
    (their running targets as they stand: inside a run they carry the in-run updates, past the run's end they do not),
    each row's path continuing from its last state (state 0 before column 0). Refit: z = E·U_BB⁻¹, the rest of the run
    updated at once, the columns after the run by one product at its end.

    Returns (before, settled, states): each column as it stood before it was settled, the settled table values (units
    of the row scale) and the trellis states."""
    import scipy.linalg as sl
    T = np.array(X, dtype=np.float64, copy=True)
    T[:, dead] = 0
    rows, n = T.shape
    values = np.asarray(values, dtype=np.float64)
    before = np.empty_like(T)
    settled = np.empty_like(T)
    states = np.empty((rows, n), dtype=np.int64)
    state = np.zeros(rows, dtype=np.int64)
    Sc = np.asarray(S, dtype=np.float64)[:, None]
    for b0 in range(0, n, lazy):
        b1 = min(b0 + lazy, n)
        Z = np.empty((rows, b1 - b0))
        for j in range(b0, b1, width):
            w = min(width, n - j)
            cols = slice(j, j + w)
            before[:, cols] = T[:, cols]
            win = np.concatenate([T[:, cols] / Sc, T[:, j + w: j + w + look] / Sc], 1)
            if on_viterbi is not None:
                on_viterbi(j, win)
            path = viterbi(win, values, L, k, start=state)[:, :w]
            state = path[:, -1]
            q = values[path]
            settled[:, cols] = q
            states[:, cols] = path
            E = T[:, cols] - q * Sc
            z = sl.solve_triangular(U[cols, cols], E.T, lower=False, trans="T").T  # z·U_BB = E
            T[:, j + w: b1] -= z @ U[cols, j + w: b1]
            Z[:, j - b0: j - b0 + w] = z
        if b1 < n:
            T[:, b1:] -= Z @ U[b0:b1, b1:]
    return before, settled, states


def column_trellis_sweep(X, S, U, dead, values, L: int, k: int, Tm: int, width: int = 16, lazy: int = 128):
    """`sweep` with `TrellisCode.project` (codes.py:371-378): each block's columns cut into runs of Tm consecutive
    outputs (rows), each run onto its nearest free-start trellis path. Returns (before, settled, states)."""
    import scipy.linalg as sl
    T = np.array(X, dtype=np.float64, copy=True)
    T[:, dead] = 0
    rows, n = T.shape
    values = np.asarray(values, dtype=np.float64)
    before = np.empty_like(T)
    settled = np.empty_like(T)
    states = np.empty((rows, n), dtype=np.int64)
    Sc = np.asarray(S, dtype=np.float64)[:, None]
    for b0 in range(0, n, lazy):
        b1 = min(b0 + lazy, n)
        Z = np.empty((rows, b1 - b0))
        for j in range(b0, b1, width):
            w = min(width, n - j)
            cols = slice(j, j + w)
            before[:, cols] = T[:, cols]
            xs = T[:, cols] / Sc
            seqs = xs.reshape(rows // Tm, Tm, w).transpose(0, 2, 1).reshape(-1, Tm)
            st = viterbi(seqs, values, L, k)
            st = st.reshape(rows // Tm, w, Tm).transpose(0, 2, 1).reshape(rows, w)
            q = values[st]
            settled[:, cols] = q
            states[:, cols] = st
            E = T[:, cols] - q * Sc
            z = sl.solve_triangular(U[cols, cols], E.T, lower=False, trans="T").T
            T[:, j + w: b1] -= z @ U[cols, j + w: b1]
            Z[:, j - b0: j - b0 + w] = z
        if b1 < n:
            T[:, b1:] -= Z @ U[b0:b1, b1:]
    return before, settled, states


def row_scale(X) -> np.ndarray:
    """codes.py:436: S = max(sqrt(mean_j X²), 1e-12) per row."""
    return np.maximum(np.sqrt(np.mean(np.asarray(X, dtype=np.float64) ** 2, axis=1)), 1e-12)


def ldlq_row_words(W, H, values, L: int, k: int, in_seed: int, width: int = 16, look: int = 8, lazy: int = 128):
    """`ldlq_words([W], H, RowTrellisCode(L, k, width, look), [seed], in_seed=in_seed, out_rot=False)` (codes.py:413-462)
    for one row group: X = W·R_inᵀ, S per row, Hr = R_in·H·R_inᵀ, the sweep under Environment(Hr), and the word
    W_q = diag(S)·V[states]·R_in (restrict_trellis with the sweep's projection, codes.py:406-410, 223-243).
    Returns a dict with the rotated target X, S, states, settled values, the dequantized matrix and the proxy loss."""
    W = np.asarray(W, dtype=np.float64)
    n = W.shape[1]
    R = rht(n, in_seed)
    X = W @ R.T
    S = row_scale(X)
    Hr = R @ np.asarray(H, dtype=np.float64) @ R.T
    U, dead, _ = environment(Hr)
    before, settled, states = row_trellis_sweep(X, S, U, dead, values, L, k, width, look, lazy)
    if not is_trellis_path(states, L, k):
        raise ValueError("the given projection is not a path through this trellis")
    Wq = (settled * S[:, None]) @ R
    return {"X": X, "S": S, "U": U, "Hr": Hr, "before": before, "settled": settled, "states": states, "Wq": Wq,
            "proxy": proxy_loss(Wq, W, H)}


def proxy_loss(Wq, W, H) -> float:
    """quantize.py:1324-1325: tr(ΔW·H·ΔWᵀ) = Σ (E·H) ⊙ E, E = W_q − W."""
    E = np.asarray(Wq, dtype=np.float64) - np.asarray(W, dtype=np.float64)
    return float(np.sum((E @ np.asarray(H, dtype=np.float64)) * E))


def trellis_states(values, table) -> np.ndarray:
    """quantize.py:502-510: each value's state, its index in the table (nearest of the two sorted neighbours)."""
    t = np.asarray(table, dtype=np.float64).ravel()
    order = np.argsort(t, kind="stable")
    st = t[order]
    v = np.asarray(values, dtype=np.float64)
    pos = np.clip(np.searchsorted(st, v), 1, len(st) - 1)
    pos = np.where(np.abs(v - st[pos - 1]) <= np.abs(st[pos] - v), pos - 1, pos)
    assert float(np.abs(st[pos] - v).max(initial=0.0)) < 1e-9, "a trellis value not in its table"
    return order[pos].astype(np.int16)


# ----------------------------------------------------------------------------- scalar-level LDLQ (ldlq_gpu.py:15-49)


def ldlq_factor(Hr, damp: float = 0.01) -> np.ndarray:
    """`opgraph.ldlq_gpu.ldlq_factor` (ldlq_gpu.py:15-26): H symmetrized; damping d·mean(diag H)·I for d = damp,
    10·damp, 100·damp until it factors; the upper Cholesky factor U of its inverse (Uᵀ·U = H⁻¹)."""
    H = np.asarray(Hr, dtype=np.float64)
    H = 0.5 * (H + H.T)
    mean = float(np.mean(np.diag(H)))
    for d in (damp, 10 * damp, 100 * damp):
        try:
            L = np.linalg.cholesky(H + d * mean * np.eye(len(H)))
        except np.linalg.LinAlgError:
            continue
        Li = np.linalg.inv(L)
        return np.linalg.cholesky(Li.T @ Li).T
    raise AssertionError("H is not positive definite even with damping")


def ldlq_round(X, U, levels, block: int = 128) -> np.ndarray:
    """`opgraph.ldlq_gpu.ldlq_round` (ldlq_gpu.py:29-49): every entry to a level, inputs in order within blocks of
    `block`, q = levels[number of midpoints below x], e = (x − q) / U[j][j] carried into the block's later inputs
    through U's row, then into the inputs after the block through one product."""
    X = np.array(X, dtype=np.float64)
    U = np.asarray(U, dtype=np.float64)
    lv = np.asarray(levels, dtype=np.float64)
    mids = (lv[1:] + lv[:-1]) / 2
    Q = np.empty_like(X)
    n = X.shape[1]
    for a in range(0, n, block):
        b = min(a + block, n)
        Err = np.empty((X.shape[0], b - a))
        for j in range(a, b):
            q = lv[np.searchsorted(mids, X[:, j], side="left")]
            Q[:, j] = q
            e = (X[:, j] - q) / U[j, j]
            X[:, j + 1:b] -= e[:, None] * U[j, j + 1:b][None, :]
            Err[:, j - a] = e
        X[:, b:] -= Err @ U[a:b, b:]
    return Q


# ----------------------------------------------------------------------------- statistics (quantize.py:1457-1470, 1330-1335)


def hessian_accumulate(chunks, weights=None, ref_chunks=None):
    """quantize.py:1412-1470: per calibration chunk, H += Xᵀ(w⊙X) and (QEP) D += X_refᵀ(w⊙X) in fp32 (the model's
    activations cast to fp32, the token weights fp32), n_tok counted unweighted; then H/n_tok (and D/n_tok − H) as fp64.
    `chunks` are (tokens, d) arrays. Restated with torch's fp32 CPU GEMM, the reference's own arithmetic."""
    import torch
    d = chunks[0].shape[1]
    H = torch.zeros(d, d, dtype=torch.float32)
    D = torch.zeros(d, d, dtype=torch.float32) if ref_chunks is not None else None
    n_tok = 0
    for c, x in enumerate(chunks):
        x = torch.as_tensor(x).float()
        xw = x if weights is None else x * torch.as_tensor(weights[c]).float().reshape(-1, 1)
        if D is not None:
            D += torch.as_tensor(ref_chunks[c]).float().T @ xw
        H += x.T @ xw
        n_tok += len(x)
    Hd = (H / n_tok).double().numpy()
    if D is None:
        return Hd, None
    return Hd, (D / n_tok).double().numpy() - Hd


def cross_target(H, D, alpha: float, lam: float = 0.1) -> np.ndarray:
    """quantize.py:1330-1335: M = I + α·(solve(H + λ·mean(diag H)·I, Dᵀ))ᵀ."""
    H = np.asarray(H, dtype=np.float64)
    eye = np.eye(len(H))
    return eye + alpha * np.linalg.solve(H + lam * np.mean(np.diag(H)) * eye, np.asarray(D, dtype=np.float64).T).T


# ----------------------------------------------------------------------------- packed codes (compiler_artifact.py:225-297)


def pack_symbols(q, bits: int) -> np.ndarray:
    """compiler_artifact.py:225-240: each row padded to a multiple of 32 symbols; symbol i of a group of 32 sits at
    bit i·bits of the group's `bits` little-endian uint32 words."""
    q = np.asarray(q)
    if q.ndim != 2 or not 1 <= bits <= 8 or np.any(q < 0) or np.any(q >= 1 << bits):
        raise ValueError("invalid symbols or width")
    m, n = q.shape
    q = np.pad(q, ((0, 0), (0, (-n) % 32))).astype(np.uint64).reshape(m, -1, 32)
    out = np.zeros((m, q.shape[1], bits), dtype=np.uint64)
    for i in range(32):
        word, shift = divmod(i * bits, 32)
        v = q[:, :, i] << np.uint64(shift)
        out[:, :, word] |= v & np.uint64(0xFFFFFFFF)
        if shift + bits > 32:
            out[:, :, word + 1] |= v >> np.uint64(32)
    return out.astype(np.uint32).reshape(m, -1)


def unpack_symbols(codes, bits: int, columns: int) -> np.ndarray:
    """compiler_artifact.py:243-258."""
    codes = np.asarray(codes).astype(np.uint64)
    m = codes.shape[0]
    blocks = (columns + 31) // 32
    words = codes.reshape(m, blocks, bits)
    out = np.empty((m, blocks, 32), dtype=np.uint64)
    for i in range(32):
        word, shift = divmod(i * bits, 32)
        v = words[:, :, word] >> np.uint64(shift)
        if shift + bits > 32:
            v |= words[:, :, word + 1] << np.uint64(32 - shift)
        out[:, :, i] = v & np.uint64((1 << bits) - 1)
    return out.astype(np.uint32).reshape(m, -1)[:, :columns]


def valid_path(states, bits: int, state_bits: int = 12) -> bool:
    """compiler_artifact.py:261-267: a row trellis from state zero."""
    s = np.asarray(states, dtype=np.int64)
    return (s.ndim == 2 and s.shape[1] > 0 and bool(np.all((s >= 0) & (s < (1 << state_bits))))
            and bool(np.all(s[:, 0] < (1 << bits)))
            and bool(np.all(s[:, 1:] >> bits == s[:, :-1] & ((1 << (state_bits - bits)) - 1))))


def pack_trellis(states, bits: int, state_bits: int = 12) -> np.ndarray:
    """compiler_artifact.py:276-284: symbols = state & (2^k − 1), padded forward to 32, reversed, packed."""
    s = np.asarray(states, dtype=np.int64)
    if not valid_path(s, bits, state_bits):
        raise ValueError("states are not a row trellis from zero")
    sym = s & ((1 << bits) - 1)
    sym = np.pad(sym, ((0, 0), (0, (-sym.shape[1]) % 32)))
    return pack_symbols(sym[:, ::-1], bits)


def unpack_trellis(codes, bits: int, columns: int, state_bits: int = 12) -> np.ndarray:
    """compiler_artifact.py:287-297: unpack, reverse, and shift the symbols back into 12-bit states."""
    padded = (columns + 31) // 32 * 32
    sym = unpack_symbols(codes, bits, padded)[:, ::-1]
    state = np.zeros(len(sym), dtype=np.uint32)
    out = np.empty((len(sym), columns), dtype=np.uint32)
    mask = (1 << state_bits) - 1
    for i in range(columns):
        state = ((state << bits) | sym[:, i]) & mask
        out[:, i] = state
    return out


def decode_rotated_groups(groups, shape, columns: int, state_bits: int = 12) -> np.ndarray:
    """compiler_artifact.py:433-442 for trellis groups: groups = [(rows, codes, bits, scales, table)] → fp32 table·scale
    values (before the input transform)."""
    out = np.empty(shape, dtype=np.float32)
    for rows, codes, bits, scales, table in groups:
        idx = unpack_trellis(codes, bits, columns, state_bits)
        out[np.asarray(rows, dtype=np.int64)] = np.asarray(table, np.float32)[idx] * np.asarray(scales, np.float32)[:, None]
    return out
