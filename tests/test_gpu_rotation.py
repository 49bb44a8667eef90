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


@pytest.mark.parametrize("n", [64, 200, 960, 2560, 4096, 9728])
def test_few_rows_equal_the_one_row_per_cta_form(n):
    """Fewer than 128 rows take the split form (many CTAs per row, two launches); its results equal those of the
    one-CTA-per-row form bit for bit, both directions, out of place and in place."""
    from lookatmyquant_b200.rotation import Rotation
    rot = Rotation(n, 17, "cuda")
    M = torch.randn(160, n, dtype=torch.float64, generator=torch.Generator().manual_seed(n)).cuda()
    for run in (rot.rows, rot.rows_t):
        whole = run(M)  # 160 rows: one CTA per row
        for k in (1, 5, 127):
            assert torch.equal(run(M[:k]), whole[:k])
            inplace = M[:k].clone()
            run(inplace, out=inplace)
            assert torch.equal(inplace, whole[:k])


@pytest.mark.parametrize("n", [960, 2560, 4096, 9728, 200])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_activation_rotation_matches_fp64(n, dtype):
    """lamq_rht_rows_act (fp32 sums, bf16/fp32 in and out) against the fp64 rotation: R x and Rᵀ x to fp32 (or bf16)
    rounding."""
    from lookatmyquant_b200.rotation import Rotation
    R = Rotation(n, 301)
    x = torch.randn(300, n, generator=torch.Generator().manual_seed(n)).to(dtype).cuda()
    want = R.rows(x.double())
    for out_dtype, tol in ((torch.float32, 1e-5), (torch.bfloat16, 1e-2)):
        got = R.rows_act(x, out_dtype)
        assert got.dtype == out_dtype and got.shape == (300, n)
        assert (got.double() - want).abs().max() <= tol * want.abs().max()
    want_t = R.rows_t(x.double())
    got_t = R.rows_t_act(x, torch.float32)
    assert (got_t.double() - want_t).abs().max() <= 1e-5 * want_t.abs().max()
