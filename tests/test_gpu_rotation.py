"""GPU parity: the factored randomized Hadamard transforms against the reference's dense rht (oracle, pinned by the
golden rotations)."""

import numpy as np
import pytest
import torch

from oracle import core as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n,seed", [(64, 5), (200, 7), (256, 301), (320, 9), (960, 301), (2560, 1301),
                                    (4096, 2201), (9728, 3301)])
def test_rows_and_transpose(n, seed):
    from lookatmyquant_b200.rotation import Rotation
    R = O.rht(n, seed)
    rot = Rotation(n, seed, "cuda")
    M = np.random.default_rng(n).standard_normal((37, n))
    Mt = torch.as_tensor(M).cuda()
    got = rot.rows(Mt).cpu().numpy()
    assert np.abs(got - M @ R.T).max() < 1e-12 * np.abs(M).max() * np.sqrt(n)
    got_t = rot.rows_t(Mt).cpu().numpy()
    assert np.abs(got_t - M @ R).max() < 1e-12 * np.abs(M).max() * np.sqrt(n)


@pytest.mark.parametrize("n", [256, 960, 2560])
def test_conjugation(n):
    from lookatmyquant_b200.rotation import Rotation
    R = O.rht(n, 11)
    A = np.random.default_rng(1).standard_normal((3 * n, n))
    H = A.T @ A / (3 * n)
    got = Rotation(n, 11, "cuda").conj(torch.as_tensor(H).cuda()).cpu().numpy()
    ref = R @ H @ R.T
    assert np.abs(got - ref).max() < 1e-12 * np.abs(ref).max()
