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
