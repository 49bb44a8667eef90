"""GPU parity of the fp64 tensor-core linear algebra: GEMM, Cholesky inverse, the environment factor U (against the
oracle's restatement of frame.py:515-522, itself pinned by the reference's golden U) and the QEP target (against
quantize.py:1330-1335 restated)."""

import numpy as np
import pytest
import torch

from oracle import core as O

pytestmark = pytest.mark.gpu


def spd(n, seed, tokens=None):
    rng = np.random.default_rng(seed)
    A = rng.standard_normal((tokens or 2 * n, n)) * np.exp(rng.standard_normal(n))
    return A.T @ A / len(A)


# the shapes reach every CTA tile: 32 x 32 (the first three), 64 x 64 (1024 x 512) and 128 x 128 (2048 x 1100)
@pytest.mark.parametrize("M,N,K", [(1, 1, 1), (130, 70, 17), (257, 300, 129), (1024, 512, 640), (2048, 1100, 300)])
@pytest.mark.parametrize("transB", [False, True])
def test_gemm(M, N, K, transB):
    from lookatmyquant_b200.linalg import gemm
    rng = np.random.default_rng(M + N + K)
    A = rng.standard_normal((M, K))
    B = rng.standard_normal((N, K) if transB else (K, N))
    C = rng.standard_normal((M, N))
    got = gemm(torch.as_tensor(A).cuda(), torch.as_tensor(B).cuda(), C=torch.as_tensor(C).cuda(), transB=transB,
               alpha=-0.5, beta=2.0).cpu().numpy()
    ref = -0.5 * (A @ (B.T if transB else B)) + 2.0 * C
    assert np.abs(got - ref).max() < 1e-12 * np.abs(ref).max() * np.sqrt(K)


@pytest.mark.parametrize("M,N,K", [(100, 90, 33), (1500, 1400, 77)])
def test_gemm_unaligned_rows(M, N, K):
    """Operands whose rows start off a 16-byte boundary (odd leading dimension): the 8-byte copy path."""
    from lookatmyquant_b200.linalg import gemm
    rng = np.random.default_rng(M)
    A = torch.as_tensor(rng.standard_normal((M, K + 1))).cuda()[:, 1:]
    B = torch.as_tensor(rng.standard_normal((K, N + 1))).cuda()[:, 1:]
    got = gemm(A, B).cpu().numpy()
    ref = A.cpu().numpy() @ B.cpu().numpy()
    assert np.abs(got - ref).max() < 1e-12 * np.abs(ref).max() * np.sqrt(K)


@pytest.mark.parametrize("n", [1, 33, 65, 100, 128, 300, 1024, 2560])
def test_cholesky_inverse(n):
    from lookatmyquant_b200.linalg import cholesky_inverse_lower
    H = spd(n, n) + 0.01 * np.eye(n)
    X = cholesky_inverse_lower(torch.as_tensor(H).cuda()).cpu().numpy()
    assert np.allclose(np.triu(X, 1), 0)
    L = np.linalg.cholesky(H)
    assert np.abs(X @ L - np.eye(n)).max() < 1e-9


def test_environment_matches_reference_golden(golden):
    from lookatmyquant_b200.linalg import env_factor
    g = golden("environment")
    U, dead, check = env_factor(torch.as_tensor(g["H"].astype(np.float64)).cuda())
    check()
    assert np.array_equal(dead.cpu().numpy(), g["dead"])
    assert np.abs(U.cpu().numpy() - g["U"]).max() <= 1e-10 * np.abs(g["U"]).max()


@pytest.mark.parametrize("n", [960, 2560, 4096])
def test_environment_matches_oracle(n):
    from lookatmyquant_b200.linalg import env_factor
    H = spd(n, 3 * n)
    U, _, check = env_factor(torch.as_tensor(H).cuda())
    check()
    Uo, _, _ = O.environment(H)
    assert np.abs(U.cpu().numpy() - Uo).max() <= 1e-9 * np.abs(Uo).max()


def test_not_positive_definite_raises():
    from lookatmyquant_b200.linalg import cholesky_inverse_lower
    H = -np.eye(64)
    with pytest.raises(AssertionError, match="not positive definite"):
        cholesky_inverse_lower(torch.as_tensor(H).cuda())


@pytest.mark.parametrize("n,rows", [(256, 1000), (512, 100), (300, 77), (200, 500)])
def test_cross_target(n, rows):
    from lookatmyquant_b200.linalg import CrossTarget
    H = spd(n, 7)
    D = 0.01 * np.random.default_rng(8).standard_normal((n, n))
    W = 0.02 * np.random.default_rng(9).standard_normal((rows, n))
    M = O.cross_target(H, D, 0.5, 0.1)
    ct = CrossTarget(torch.as_tensor(H).cuda(), torch.as_tensor(D).cuda(), 0.5, 0.1, rows=rows)
    got = ct.apply(torch.as_tensor(W).cuda()).cpu().numpy()
    ref = W @ M
    assert np.abs(got - ref).max() <= 1e-11 * np.abs(ref).max()
