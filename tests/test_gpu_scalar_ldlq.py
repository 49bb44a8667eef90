"""The scalar-level LDLQ of opgraph/ldlq_gpu.py (ldlq_factor, ldlq_round) and the generic sweep of
opgraph/syntax.py:86-124 on the GPU, against the reference's own outputs (tests/golden/ldlq_gpu.npz)."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_ldlq_factor_matches_reference(golden):
    from lookatmyquant_b200.ldlq_gpu import ldlq_factor
    g = golden("ldlq_gpu")
    for H, U in ((g["H"], g["U"]), (g["Hbad"], g["Ubad"])):  # the second one needs the 10x damping
        got = ldlq_factor(torch.as_tensor(H).cuda()).cpu().numpy()
        assert np.abs(got - U).max() <= 1e-11 * np.abs(U).max()


def test_ldlq_factor_raises_like_reference():
    from lookatmyquant_b200.ldlq_gpu import ldlq_factor
    H = -torch.eye(16, dtype=torch.float64).cuda()
    with pytest.raises(AssertionError, match="not positive definite even with damping"):
        ldlq_factor(H)


@pytest.mark.parametrize("nl,block", [(8, 128), (16, 48)])
def test_ldlq_round_matches_reference(golden, nl, block):
    from lookatmyquant_b200.ldlq_gpu import ldlq_round
    g = golden("ldlq_gpu")
    Q = ldlq_round(torch.as_tensor(g["X"]).cuda(), torch.as_tensor(g["U"]).cuda(), torch.as_tensor(g[f"levels{nl}"]),
                   block=block).cpu().numpy()
    ref = g[f"Q{nl}_b{block}"]
    assert (Q == ref).mean() >= 0.999  # the products after each block sum in another order than the CPU's
    assert set(np.unique(Q)) <= set(g[f"levels{nl}"])


def test_ldlq_round_large_matches_oracle():
    """A 1000 x 2560 rounding (20 blocks) against the oracle's restatement."""
    from lookatmyquant_b200.ldlq_gpu import ldlq_factor, ldlq_round
    from oracle import core as O
    rng = np.random.default_rng(3)
    n = 2560
    A = rng.standard_normal((2 * n, n)) * np.exp(0.5 * rng.standard_normal(n))
    H = A.T @ A / (2 * n)
    X = rng.standard_normal((1000, n))
    lv = np.sort(rng.standard_normal(8))
    U = ldlq_factor(torch.as_tensor(H).cuda())
    Q = ldlq_round(torch.as_tensor(X).cuda(), U, torch.as_tensor(lv)).cpu().numpy()
    ref = O.ldlq_round(X, U.cpu().numpy(), lv)
    assert (Q == ref).mean() >= 0.999


@pytest.mark.parametrize("width", [1, 4])
def test_generic_sweep_matches_reference(golden, width):
    from lookatmyquant_b200 import syntax
    from lookatmyquant_b200.frame import Environment
    g = golden("ldlq_gpu")
    Hd = g["H"].copy()
    Hd[5, :] = 0
    Hd[:, 5] = 0
    env = Environment(torch.as_tensor(Hd).cuda())
    lv = torch.as_tensor(g["levels8"]).cuda()
    mids = (lv[1:] + lv[:-1]) / 2

    def nearest(j, cols, T):
        return lv[torch.bucketize(cols.contiguous(), mids)]
    got = syntax.sweep(torch.as_tensor(g["X"]).cuda(), env, nearest, width=width, lazy=64).cpu().numpy()
    ref = g[f"sweep_w{width}"]
    assert np.abs(got - ref).max() <= 1e-10 * np.abs(ref).max()
