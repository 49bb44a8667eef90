"""The oracle against the reference's own outputs (golden vectors made by tests/golden/make_golden.py)."""

import sys
import numpy as np
import pytest
import torch

from conftest import GOLDEN, table
from oracle import core as O


@pytest.mark.parametrize("k", [1, 2, 3, 4])
def test_viterbi_matches_reference(golden, k):
    g = golden("viterbi")
    v = table(k)
    assert np.array_equal(O.viterbi(g[f"k{k}_X"], v, 12, k, start=g[f"k{k}_start"]), g[f"k{k}_states_start"])
    assert np.array_equal(O.viterbi(g[f"k{k}_Xfree"], v, 12, k), g[f"k{k}_states_free"])
    zero = np.zeros(len(g[f"k{k}_Xshort"]), dtype=np.int64)
    assert np.array_equal(O.viterbi(g[f"k{k}_Xshort"], v, 12, k, start=zero), g[f"k{k}_states_short"])


def test_viterbi_small_tables(golden):
    g = golden("viterbi")
    assert np.array_equal(O.viterbi(g["L8_X"], g["L8_values"], 8, 2), g["L8_states"])
    assert np.array_equal(O.viterbi(g["L4_X"], g["L4_values"], 4, 1), g["L4_states"])


def test_viterbi_is_optimal():
    """As tests/test_codes.py:101-117 of the reference: the decoded path is the brute-force minimum (L=4, k=1, T=7)."""
    rng = np.random.default_rng(0)
    v = rng.standard_normal(16).astype(np.float32).astype(np.float64)
    X = rng.standard_normal((5, 7)).astype(np.float32).astype(np.float64)
    st = O.viterbi(X, v, 4, 1)
    assert O.is_trellis_path(st, 4, 1)
    got = ((X - v[st]) ** 2).sum(1)
    for r in range(len(X)):
        assert abs(got[r] - O.viterbi_bruteforce(X[r], v, 4, 1)) < 1e-4


def test_empty_and_single_column():
    v = table(2)
    assert O.viterbi(np.zeros((0, 5)), v, 12, 2).shape == (0, 5)
    x = np.array([[0.3], [-1.2]])
    st = O.viterbi(x, v, 12, 2)
    assert np.array_equal(st[:, 0], np.argmin((x.astype(np.float32) - v.astype(np.float32)) ** 2, axis=1))


@pytest.mark.parametrize("n", [64, 200, 256, 320, 960, 2560, 4096, 9728])
def test_rotations_match_reference(golden, n):
    g = golden("rotation")
    A, B = O.hadamard_factors(n)
    assert (A.shape[0], B.shape[0]) == tuple(g[f"n{n}_shapes"])
    R = O.rht(n, int(g[f"n{n}_seed"]))
    assert np.array_equal(R[:2], g[f"n{n}_rows"])
    vec = torch.randn(n, generator=torch.Generator().manual_seed(n), dtype=torch.float64).numpy()
    assert np.abs(R @ vec - g[f"n{n}_Rv"]).max() < 1e-12
    if n <= 2560:
        assert np.abs(R @ R.T - np.eye(n)).max() < 1e-10


def test_environment_matches_reference(golden):
    g = golden("environment")
    U, dead, _ = O.environment(g["H"].astype(np.float64))
    assert np.array_equal(dead, g["dead"])
    assert np.abs(U - g["U"]).max() <= 1e-12 * np.abs(g["U"]).max()


@pytest.mark.parametrize("case", ["a", "b", "c", "d"])
def test_ldlq_row_words_match_reference(golden, case):
    g = golden("ldlq_row")
    m, n, k, seed, in_seed = (int(x) for x in g[f"{case}_meta"])
    out = O.ldlq_row_words(g[f"{case}_W"].astype(np.float64), g[f"{case}_H"].astype(np.float64), table(k), 12, k,
                           in_seed)
    assert np.array_equal(out["states"], g[f"{case}_states"])
    assert np.abs(out["S"] - g[f"{case}_S"]).max() < 1e-15
    assert np.abs(out["Wq"] - g[f"{case}_Wq"]).max() < 1e-7  # the fixture is stored in fp32
    assert abs(out["proxy"] - float(g[f"{case}_proxy"])) <= 1e-12 * abs(float(g[f"{case}_proxy"]))
    assert np.array_equal(O.pack_trellis(out["states"], k), g[f"{case}_packed"])
    assert np.array_equal(O.unpack_trellis(g[f"{case}_packed"], k, n), out["states"])


def test_ldlq_without_rotation_dead_inputs(golden):
    g = golden("ldlq_row")
    m, n, k = (int(x) for x in g["e_meta"][:3])
    W, H = g["e_W"].astype(np.float64), g["e_H"].astype(np.float64)
    S = O.row_scale(W)
    U, dead, _ = O.environment(H)
    assert dead.sum() == 2
    _, settled, states = O.row_trellis_sweep(W, S, U, dead, table(k), 12, k)
    assert np.array_equal(states, g["e_states"])
    assert np.abs(settled * S[:, None] - g["e_Wq"]).max() < 1e-7


def test_row_groups_match_reference(golden):
    """quantize.quantize_row_groups (quantize.py:530-565): groups swept separately, states offset by 4096 per table."""
    g = golden("row_groups")
    W, H, perm = g["W"].astype(np.float64), g["H"].astype(np.float64), g["perm"]
    groups = [(perm[i * 64:(i + 1) * 64], int(b)) for i, b in enumerate(g["bits"])]
    in_seed = int(g["in_seed"])
    states = np.empty(W.shape, dtype=np.int64)
    for ti, (rows, bits) in enumerate(groups):
        out = O.ldlq_row_words(W[rows], H, table(bits), 12, bits, in_seed)
        states[rows] = out["states"] + 4096 * ti
    assert np.array_equal(states, g["states"])


def test_column_trellis_matches_reference(golden):
    """TrellisCode (codes.py:363-383), the `measure` path with a two-sided rotation."""
    g = golden("column_trellis")
    m, n, k, seed, Tm = (int(x) for x in g["meta"])
    W, H = g["W"].astype(np.float64), g["H"].astype(np.float64)
    Ri, Ro = O.rht(n, seed + 1), O.rht(m, seed)
    X = Ro @ W @ Ri.T
    S = O.row_scale(X)
    U, dead, _ = O.environment(Ri @ H @ Ri.T)
    _, settled, states = O.column_trellis_sweep(X, S, U, dead, table(k), 12, k, Tm)
    assert np.array_equal(settled, g["settled"])
    Wq = Ro.T @ (settled * S[:, None]) @ Ri
    assert np.abs(Wq - g["Wq"]).max() < 1e-7


def test_pack_symbols_round_trip():
    rng = np.random.default_rng(1)
    for bits in (1, 2, 3, 4, 5, 8):
        q = rng.integers(0, 1 << bits, size=(7, 45))
        assert np.array_equal(O.unpack_symbols(O.pack_symbols(q, bits), bits, 45), q)


def test_trellis_states_inverts_table():
    v = table(3)
    st = np.random.default_rng(2).integers(0, 4096, size=(4, 9))
    assert np.array_equal(O.trellis_states(v[st], v), st.astype(np.int16))


def test_packed_artifact_matches_reference(golden):
    """The reference's own encode_entry and decode_rotated (compiler_artifact.py:307-360, :433-442) on row groups."""
    g = golden("artifact")
    groups = []
    for i in range(4):
        rows, bits = g[f"g{i}_rows"].astype(np.int64), int(g[f"g{i}_bits"])
        ti = int(g["states"][rows[0], 0]) // 4096
        states = g["states"][rows].astype(np.int64) - 4096 * ti
        assert np.array_equal(O.pack_trellis(states, bits), g[f"g{i}_codes"])
        assert np.array_equal(O.unpack_trellis(g[f"g{i}_codes"], bits, 200), states)
        groups.append((rows, g[f"g{i}_codes"], bits, g[f"g{i}_scales"], g["table"][4096 * ti:4096 * (ti + 1)]))
    assert np.array_equal(O.decode_rotated_groups(groups, (200, 200), 200), g["decoded"])
    import torch
    u = torch.rand(200, generator=torch.Generator().manual_seed(int(g["in_seed"])), dtype=torch.float64).numpy()
    assert np.array_equal(g["signs"], np.where(u < .5, -1, 1).astype(np.int8))


def test_oracle_viterbi_near_tie(golden):
    """The near-tie sequence of tests/golden/viterbi_neartie.npz: the oracle's separately rounded fp32 costs choose the
    reference's path."""
    g = golden("viterbi_neartie")
    assert np.array_equal(O.viterbi(g["X"], g["values"], 12, int(g["k"])), g["states"])


def test_oracle_scalar_ldlq_matches_reference(golden):
    """ldlq_gpu.ldlq_factor / ldlq_round (ldlq_gpu.py:15-49) restated, against the reference's own outputs."""
    g = golden("ldlq_gpu")
    assert np.abs(O.ldlq_factor(g["H"]) - g["U"]).max() <= 1e-12 * np.abs(g["U"]).max()
    assert np.abs(O.ldlq_factor(g["Hbad"]) - g["Ubad"]).max() <= 1e-12 * np.abs(g["Ubad"]).max()
    for nl, block in ((8, 128), (16, 48)):
        assert np.array_equal(O.ldlq_round(g["X"], g["U"], g[f"levels{nl}"], block), g[f"Q{nl}_b{block}"])


# ---- statistics, QEP and KL against the reference's own outputs (statistics.npz, kl.npz by make_golden.py)

def _stat_inputs(golden, name):
    sys.path.insert(0, str(GOLDEN))
    import statgen
    xq, xr, w, W = statgen.stat_inputs(name)
    if statgen.digest(xq + (xr or []) + (w or [])) != str(golden("statistics")[f"{name}_digest"]):
        pytest.skip("torch's CPU generator drew different inputs here than where the golden vectors were made")
    return xq, xr, w, W


def test_oracle_statistics_match_reference_covariance(golden):
    """frame.covariance (opgraph/frame.py:498-505): Σ x xᵀ of bf16 activations; the oracle's H·n_tok equals it to fp32
    accumulation error (the reference sums 8192-token fp32 chunks in fp64, the oracle per given chunk)."""
    g = golden("statistics")
    xq, _, _, _ = _stat_inputs(golden, "cov")
    H, _ = O.hessian_accumulate([x.float().numpy() for x in xq])
    ref = g["cov_cov"] / float(g["cov_ntok"])
    assert np.linalg.norm(H - ref) <= 1e-6 * np.linalg.norm(ref)


@pytest.mark.parametrize("name", ["qep", "qep_wide"])
def test_oracle_weighted_statistics_and_qep_match_reference(golden, name):
    """quantize_stage's weighted H, D (quantize.py:1457-1470) and the QEP target W·M (:1330-1335, :1482, :1503), run
    by make_golden.py statement by statement from the reference's source: the oracle agrees to fp32 rounding on H
    and D + H, and to 1e-9 on M and W·M from the golden H and D."""
    g = golden("statistics")
    xq, xr, w, W = _stat_inputs(golden, name)
    H, D = O.hessian_accumulate([x.float().numpy() for x in xq], [t.numpy() for t in w],
                                [x.float().numpy() for x in xr])
    gH, gD = g[f"{name}_H"], g[f"{name}_D"]
    assert np.linalg.norm(H - gH) <= 1e-6 * np.linalg.norm(gH)
    assert np.linalg.norm((D + H) - (gD + gH)) <= 1e-6 * np.linalg.norm(gH)
    M = O.cross_target(gH, gD, float(g["alpha"]), float(g["lam"]))
    if f"{name}_M" in g:
        assert np.abs(M - g[f"{name}_M"]).max() <= 1e-9
    tgt = g[f"{name}_target"]
    assert np.abs(W.numpy() @ M - tgt).max() <= 1e-9 * np.abs(tgt).max()


def test_kl_fixture_formula(golden):
    """quantize.evaluate's KL (quantize.py:903-920) is the mean over positions of the per-position KL recorded with it
    (the formula of compiler.py:180-187 with unit weights), and the probe is far from the floor."""
    g = golden("kl")
    assert abs(float(g["kl_pos"].astype(np.float64).mean()) - float(g["kl"])) <= 1e-6
    assert float(g["kl"]) > 0.1


def test_oracle_viterbi_on_fewer_states(golden):
    """The C restatement at L = 5..11 against the reference's viterbi (small_l.npz)."""
    g = golden("small_l")
    for c in "abcde":
        L, k, with_start = (int(v) for v in g[f"v{c}_meta"])
        out = O.viterbi(g[f"v{c}_X"], g[f"v{c}_values"], L, k, start=g[f"v{c}_start"] if with_start else None)
        assert np.array_equal(out, g[f"v{c}_states"]), c
