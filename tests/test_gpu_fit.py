"""Table fits on the GPU (codes.py:187-220) against the reference's own trellis_values fits (tests/golden/fit.npz):
the same Gaussian samples, the GPU Viterbi's states (identical to the reference's) and the same fp64 updates give
the same table."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("k", [2, 3])
@pytest.mark.parametrize("fit,seed,refine", [("ema", 5, 1), ("lloyd", 6, 2)])
def test_fit_matches_reference(golden, k, fit, seed, refine):
    from lookatmyquant_b200 import codes
    g = golden("fit")
    v = codes.fit_trellis_values(12, k, 64, seed=seed, refine=refine, fit=fit).numpy()
    ref = g[f"{fit}_k{k}"]
    assert np.abs(v - ref).max() <= 1e-12 * np.abs(ref).max()



def test_full_fit_reproduces_the_shipped_table():
    """The whole e-means fit (16·384 batches) of the k = 2, T = 256 table reproduces the reference's shipped table bit
    for bit — so the T = 320 tables fitted the same way are the reference's."""
    from lookatmyquant_b200 import codes
    v = codes.fit_trellis_values(12, 2, 256).numpy()
    shipped = np.fromfile(codes.TABLES / "trellis_L12_k2_T256_s0_ema.f64", dtype="<f8")
    assert np.array_equal(v, shipped)
