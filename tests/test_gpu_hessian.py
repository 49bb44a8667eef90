"""GPU parity: the tcgen05 Hessian / QEP-moment accumulation against the reference's fp32 expressions
(quantize.py:1457-1470, restated in oracle.core.hessian_accumulate). Bar (north star): 1e-5 relative Frobenius."""

import numpy as np
import pytest
import torch

from oracle import core as O

pytestmark = pytest.mark.gpu


def acts(tokens, d, seed, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    std = torch.exp(torch.randn(d, generator=g))
    return (torch.randn(tokens, d, generator=g) * std).to(dtype)


def weights(tokens, seed, p=0.08, big=10.0):
    g = torch.Generator().manual_seed(seed)
    return torch.where(torch.rand(tokens, generator=g) < p, big, 1.0).float()


def rel(a, b):
    return float(np.linalg.norm(np.asarray(a) - np.asarray(b)) / np.linalg.norm(np.asarray(b)))


@pytest.mark.parametrize("tokens,d", [(64, 128), (1000, 256), (5000, 200), (4096, 960)])
def test_unweighted_h(tokens, d):
    from lookatmyquant_b200.hessian import hessian
    X = acts(tokens, d, d + tokens)
    H, _ = hessian(X.cuda())
    ref, _ = O.hessian_accumulate([X.float().numpy()])
    assert rel(H.cpu().numpy(), ref) < 1e-5
    Hc = H.cpu().numpy()
    assert np.array_equal(Hc, Hc.T)


@pytest.mark.parametrize("kind", ["two values", "three values", "many values"])
@pytest.mark.parametrize("tokens,d", [(3000, 256), (20000, 512)])
def test_weighted_h_and_qep_d(tokens, d, kind):
    """Weighted tokens gathered per weight value (few distinct weights) or split into bf16 hi + lo (many)."""
    from lookatmyquant_b200.hessian import hessian
    X = acts(tokens, d, 1)
    Xr = (X.float() + 0.05 * acts(tokens, d, 2, torch.float32)).to(torch.bfloat16)
    w = weights(tokens, 3)
    g = torch.Generator().manual_seed(4)
    if kind == "three values":
        w = torch.where(torch.rand(tokens, generator=g) < 0.3, 0.25, w)
    elif kind == "many values":
        w = torch.where(w != 1.0, 1.0 + 9.0 * torch.rand(tokens, generator=g), w)
    H, D = hessian(X.cuda(), w.cuda(), Xr.cuda(), chunk_tokens=4096)
    refH, refD = O.hessian_accumulate([X.float().numpy()], [w.numpy()], [Xr.float().numpy()])
    assert rel(H.cpu().numpy(), refH) < 1e-5
    # D is a small difference of large moments: compare D + H (the accumulated moment) at the 1e-5 bar, and D itself
    assert rel((D + H).cpu().numpy(), refD + refH) < 1e-5
    assert rel(D.cpu().numpy(), refD) < 1e-3


def test_chunks_accumulate_like_one_pass():
    from lookatmyquant_b200.hessian import Statistics
    X = acts(6000, 256, 9)
    w = weights(6000, 10)
    st = Statistics(256, device="cuda")
    for a in range(0, 6000, 2048):
        st.add(X[a:a + 2048].cuda(), w[a:a + 2048].cuda())
    H, _ = st.finalize()
    st.check_status()
    ref, _ = O.hessian_accumulate([X[a:a + 2048].float().numpy() for a in range(0, 6000, 2048)],
                                  [w[a:a + 2048].numpy() for a in range(0, 6000, 2048)])
    assert rel(H.cpu().numpy(), ref) < 1e-5


def test_config2_scale_against_fp64():
    """d = 2560, 131072 tokens (a sixth of config 2's), weighted: against an fp64 computation on the GPU."""
    from lookatmyquant_b200.hessian import hessian
    from lookatmyquant_b200.workloads import activations_bf16, token_weights
    X = activations_bf16(131072, 2560, seed=5, device="cuda")
    w = token_weights(131072, seed=6, device="cuda")
    H, _ = hessian(X, w)
    Xd = X.double()
    ref = (Xd.T @ (Xd * w.double()[:, None])) / X.shape[0]
    assert float(torch.linalg.norm(H - ref) / torch.linalg.norm(ref)) < 1e-5


# ---- against the reference's own outputs (tests/golden/statistics.npz, made by make_golden.py from the reference)

def _stat_inputs(golden, name):
    import sys
    from conftest import GOLDEN
    sys.path.insert(0, str(GOLDEN))
    import statgen
    xq, xr, w, W = statgen.stat_inputs(name)
    if statgen.digest(xq + (xr or []) + (w or [])) != str(golden("statistics")[f"{name}_digest"]):
        pytest.skip("torch's CPU generator drew different inputs here than where the golden vectors were made")
    return xq, xr, w, W


def test_h_matches_reference_covariance(golden):
    """frame.covariance (opgraph/frame.py:498-505) of 27,000 bf16 tokens: H·n_tok to 1e-5 relative Frobenius."""
    from lookatmyquant_b200.hessian import Statistics
    g = golden("statistics")
    xq, _, _, _ = _stat_inputs(golden, "cov")
    st = Statistics(xq[0].shape[1], device="cuda")
    for x in xq:
        st.add(x.cuda())
    H, _ = st.finalize(n_tok=1)
    st.check_status()
    assert rel(H.cpu().numpy(), g["cov_cov"]) < 1e-5


@pytest.mark.parametrize("name", ["qep", "qep_wide"])
def test_weighted_statistics_and_qep_target_match_reference(golden, name):
    """quantize_stage's token-weighted H and D over three chunks (quantize.py:1457-1470) and the QEP target W·M
    (:1330-1335, :1482, :1503), all by the reference's own statements in make_golden.py: H and D + H to 1e-5,
    W·M from the golden H, D to 1e-10, and W·M from this build's own H, D to 1e-4 (D is a 10 % difference of
    fp32-accumulated moments)."""
    from lookatmyquant_b200.hessian import Statistics
    from lookatmyquant_b200.linalg import CrossTarget
    g = golden("statistics")
    xq, xr, w, W = _stat_inputs(golden, name)
    st = Statistics(xq[0].shape[1], cross=True, device="cuda")
    for a, b, t in zip(xq, xr, w):
        st.add(a.cuda(), t.cuda(), b.cuda())
    H, D = st.finalize()
    st.check_status()
    gH, gD, tgt = g[f"{name}_H"], g[f"{name}_D"], g[f"{name}_target"]
    assert rel(H.cpu().numpy(), gH) < 1e-5
    assert np.linalg.norm((D + H).cpu().numpy() - (gD + gH)) < 1e-5 * np.linalg.norm(gH)
    alpha, lam = float(g["alpha"]), float(g["lam"])
    for rows in (W.shape[0], 10 * W.shape[1]):  # W + α((W·D)·Lc⁻ᵀ)·Lc⁻¹, and M formed once
        ct = CrossTarget(torch.as_tensor(gH).cuda(), torch.as_tensor(gD).cuda(), alpha, lam, rows=rows)
        got = ct.apply(W.cuda()).cpu().numpy()
        ct.check()
        assert np.abs(got - tgt).max() <= 1e-10 * np.abs(tgt).max()
    ct = CrossTarget(H, D, alpha, lam, rows=W.shape[0])
    got = ct.apply(W.cuda()).cpu().numpy()
    assert rel(got, tgt) < 1e-4


def test_config2_d9728_token_subset_against_oracle():
    """Config 2's second pass (d = 9728, token weights 10 on Bernoulli(0.08)) on 8192 tokens: the tcgen05 paired
    kernel against the oracle's fp32 accumulation (quantize.py:1457-1470) at the 1e-5 bar."""
    from lookatmyquant_b200.hessian import hessian
    from lookatmyquant_b200.workloads import activations_bf16, token_weights
    X = activations_bf16(8192, 9728, seed=21, device="cuda")
    w = token_weights(8192, seed=22, device="cuda")
    H, _ = hessian(X, w)
    ref, _ = O.hessian_accumulate([X.float().cpu().numpy()], [w.cpu().numpy()])
    assert rel(H.cpu().numpy(), ref) < 1e-5


@pytest.mark.parametrize("tokens,d,chunk", [(100000, 256, 4096), (131072, 2560, 8192), (32768, 9728, 4096)])
def test_statistics_are_bit_reproducible(tokens, d, chunk):
    """Each tile's chunks are added into the fp32 accumulators in chunk order, whichever CTAs computed them: three runs
    give the same bits. The shapes take every schedule: all units in one wave with a tile's chunks side by side
    (d = 256), tiles fewer than CTA pairs (d = 2560), and full windows plus a partial last one (d = 9728)."""
    from lookatmyquant_b200.hessian import Statistics
    X, Xr = acts(tokens, d, 11).cuda(), acts(tokens, d, 12).cuda()
    w = weights(tokens, 13).cuda()
    runs = []
    for _ in range(3):
        st = Statistics(d, cross=True, device="cuda", chunk_tokens=chunk)
        st.add(X, w, Xr)
        torch.cuda.synchronize()
        st.check_status()
        runs.append((st.accH.clone(), st.accD.clone()))
        del st
    for H, D in runs[1:]:
        assert torch.equal(H, runs[0][0])
        assert torch.equal(D, runs[0][1])
