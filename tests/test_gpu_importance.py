"""Row importance (row_importance.py:57-93) and GuidedQuant token weights (quantize.py:853-894) against the reference
(tests/golden/importance.npz): the same tiny fp32 Llama (its weights from the fixture), the reference's sampled tokens
replayed; the per-channel E[g²]·E[y²] from this library's fp64 square sums against the reference's own hooks to 1e-4
relative (fp32 forward/backward on two devices), the token weights to 1e-4; the square sums against fp64 torch."""

import sys

import numpy as np
import pytest
import torch

from conftest import GOLDEN

pytestmark = pytest.mark.gpu


def _model(g):
    sys.path.insert(0, str(GOLDEN))
    import statgen
    names = list(g["state"])
    state = {k: torch.as_tensor(g[f"p{i}"]).view(torch.bfloat16).float() for i, k in enumerate(names)}
    model = statgen.tiny_llama(state=state).cuda()
    for p in model.parameters():
        p.requires_grad_(False)
    return model


@pytest.mark.parametrize("dtype,rows,cols", [(torch.float32, 1000, 300), (torch.bfloat16, 777, 2560),
                                             (torch.float32, 3, 1)])
def test_square_sums_against_fp64(dtype, rows, cols):
    from lookatmyquant_b200.importance import square_sums
    x = torch.randn(rows, cols, device="cuda").to(dtype)
    acc = torch.full((cols,), 0.5, dtype=torch.float64, device="cuda")
    r = square_sums(x, acc, rows=True)
    xd = x.double()
    assert torch.allclose(acc, 0.5 + xd.pow(2).sum(0), rtol=1e-12, atol=0)
    assert torch.allclose(r, xd.pow(2).sum(1), rtol=1e-12, atol=0)
    acc2 = torch.full((cols,), 0.5, dtype=torch.float64, device="cuda")
    square_sums(x, acc2)
    assert torch.equal(acc, acc2)  # a fixed summation order


def test_row_importance_matches_reference(golden):
    from lookatmyquant_b200.importance import importance_summary, row_importance
    g = golden("importance")
    model = _model(g)
    mods = {f"{l}.{n}": m for l, L in enumerate(model.model.layers) for n, m in L.named_modules()
            if isinstance(m, torch.nn.Linear)}
    assert list(mods) == list(g["mods"])
    sampled = [torch.as_tensor(s) for s in g["sampled"]]
    imp, drawn = row_importance(model, torch.as_tensor(g["windows"]), mods,
                                position_weight=torch.as_tensor(g["weight"]), sampled=sampled)
    for k in mods:
        want = torch.as_tensor(g[f"imp_{k}"]).cuda()
        assert torch.allclose(imp[k], want, rtol=1e-4, atol=0), k
    summ = importance_summary(imp, {k: m.weight.numel() for k, m in mods.items()})
    assert summ["median AM/GM"] >= 1.0 and "weight-averaged bits worth" in summ


def test_guided_weights_match_reference(golden):
    from lookatmyquant_b200.importance import guided_weights
    g = golden("importance")
    model = _model(g)
    mods = {f"{l}.{n}": m for l, L in enumerate(model.model.layers) for n, m in L.named_modules()
            if isinstance(m, torch.nn.Linear)}
    windows = torch.as_tensor(g["windows"])
    chunks = [windows[:2], windows[2:]]
    base = [torch.ones(2, 32), torch.ones(1, 32) * 2.0]
    draws = torch.as_tensor(g["guided_draws"])
    sampled = [[draws[0], draws[1]], [draws[2]]]
    w, _ = guided_weights(model, chunks, mods, base, 0.1, sampled=sampled)
    for k in mods:
        got = torch.cat(w[k]).cpu()
        want = torch.as_tensor(g[f"guided_{k}"])
        assert got.shape == want.shape == (3, 32)
        assert torch.allclose(got, want, rtol=1e-4, atol=1e-6), k
        assert abs(float(got.double().mean()) - 1.0) < 1e-5
