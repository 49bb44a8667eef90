"""GPU parity: the Viterbi kernel (lamq_viterbi) against the reference's golden paths and the oracle; bit-exact."""

import numpy as np
import pytest
import torch

from conftest import table
from oracle import core as O

pytestmark = pytest.mark.gpu


def gpu_viterbi(X, values, L, k, start=None):
    from lookatmyquant_b200 import codes
    X = torch.as_tensor(np.asarray(X, dtype=np.float64)).cuda()
    st = None if start is None else torch.as_tensor(np.asarray(start, dtype=np.int64)).cuda()
    return codes.viterbi(X, torch.as_tensor(np.asarray(values, dtype=np.float64)), L, k, start=st).cpu().numpy()


@pytest.mark.parametrize("k", [1, 2, 3, 4])
def test_golden_paths(golden, k):
    g = golden("viterbi")
    v = table(k)
    assert np.array_equal(gpu_viterbi(g[f"k{k}_X"], v, 12, k, g[f"k{k}_start"]), g[f"k{k}_states_start"])
    assert np.array_equal(gpu_viterbi(g[f"k{k}_Xfree"], v, 12, k), g[f"k{k}_states_free"])
    zero = np.zeros(len(g[f"k{k}_Xshort"]), dtype=np.int64)
    assert np.array_equal(gpu_viterbi(g[f"k{k}_Xshort"], v, 12, k, zero), g[f"k{k}_states_short"])


@pytest.mark.parametrize("k", [1, 2, 3, 4])
@pytest.mark.parametrize("T", [1, 2, 24, 33, 256])
def test_random_windows_match_oracle(k, T):
    rng = np.random.default_rng(100 * k + T)
    rows = 300 if T <= 33 else 40
    X = rng.standard_normal((rows, T)) * rng.uniform(0.5, 2.0, size=(rows, 1))
    start = rng.integers(0, 4096, size=rows)
    v = table(k)
    assert np.array_equal(gpu_viterbi(X, v, 12, k, start), O.viterbi(X, v, 12, k, start=start))
    assert np.array_equal(gpu_viterbi(X, v, 12, k), O.viterbi(X, v, 12, k))


def test_ties_break_like_torch():
    """Equal costs everywhere (x far outside the table's range hits +inf... and exact ties): the smallest predecessor
    and the smallest final state win, as torch.min/argmin choose."""
    v = np.zeros(4096)
    v[::2] = 1.0
    X = np.zeros((4, 10))
    X[1] = 1.0
    X[2, ::2] = 1.0
    for k in (1, 2, 3, 4):
        assert np.array_equal(gpu_viterbi(X, v, 12, k), O.viterbi(X, v, 12, k))
        assert np.array_equal(gpu_viterbi(X, v, 12, k, np.arange(4) * 1000), O.viterbi(X, v, 12, k, np.arange(4) * 1000))


def test_empty():
    assert gpu_viterbi(np.zeros((0, 24)), table(2), 12, 2).shape == (0, 24)


def test_near_tie_matches_reference(golden):
    """A 256-step sequence whose best path beats another by one fp32 ulp in the reference's separately rounded costs
    (tests/golden/viterbi_neartie.npz, states from the reference's own viterbi): a decoder whose branch cost fuses the
    square into the add picks the other path."""
    g = golden("viterbi_neartie")
    assert np.array_equal(gpu_viterbi(g["X"], g["values"], 12, int(g["k"])), g["states"])
