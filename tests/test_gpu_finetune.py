"""The fine-tuning's trellis parts (finetune_lib.py) against the reference itself (tests/golden/finetune.npz):
`rounded` — block LDLQ of three row groups with their tables under the rotated statistics, scales refitted —
and TrellisCoded's proximal re-pick of the paths. Bars: >= 99.9 % identical states (the reference rotates in fp32,
here in fp64 rounded to fp32), scales and rounded rows to 1e-5 where the states agree, the re-picked paths identical
(their costs are the reference's fp32 arithmetic)."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _setup(g):
    from lookatmyquant_b200 import codes
    from lookatmyquant_b200.finetune import RowPath, rotated_moment
    from lookatmyquant_b200.frame import Environment
    from lookatmyquant_b200.rotation import Rotation
    n = g["W"].shape[1]
    W = torch.as_tensor(g["W"]).cuda()
    H = torch.as_tensor(g["H"].astype(np.float64)).cuda()
    R = Rotation(n, int(g["in_seed"]))
    env = Environment(rotated_moment(H, R))
    perm = torch.as_tensor(g["perm"])
    groups = [(perm[32 * i:32 * (i + 1)], k, RowPath(codes.trellis_values(12, k, 256), k))
              for i, k in enumerate((1, 2, 3))]
    return W, R, env, groups


def test_rounded_matches_reference(golden):
    from lookatmyquant_b200.finetune import rounded
    g = golden("finetune")
    W, R, env, groups = _setup(g)
    scale = torch.as_tensor(g["scale0"]).cuda()
    P, states = rounded(W, R, groups, scale, env)
    same = states.numpy() == g["states"]
    assert same.mean() >= 0.999
    rows_same = same.all(1)
    assert rows_same.mean() >= 0.9
    assert np.abs(scale.cpu().numpy() - g["scale"])[rows_same].max() <= 1e-5 * np.abs(g["scale"]).max()
    Pd, Pr = P.cpu().numpy(), g["P"]
    assert np.abs(Pd - Pr)[rows_same].max() <= 1e-5 * np.abs(Pr).max()


def test_rounded_rows_subset_matches_reference(golden):
    from lookatmyquant_b200.finetune import rounded
    g = golden("finetune")
    W, R, env, groups = _setup(g)
    scale = torch.as_tensor(g["scale0"]).cuda()
    P, states = rounded(W, R, groups, scale, env, rows=torch.as_tensor(g["rows2"]))
    assert P.shape == (16, W.shape[1])
    assert (states.numpy() == g["states2"]).mean() >= 0.999
    untouched = np.setdiff1d(np.arange(len(scale)), g["rows2"])
    assert np.array_equal(scale.cpu().numpy()[untouched], g["scale0"][untouched])


def test_repick_matches_reference(golden):
    from lookatmyquant_b200 import codes
    from lookatmyquant_b200.finetune import TrellisCoded
    g = golden("finetune")
    entry = {"states": torch.as_tensor(g["entry_states"]), "scales": torch.as_tensor(g["entry_scales"]),
             "table": codes.trellis_values(12, 2, 256).float(), "in_seed": int(g["in_seed"])}
    tc = TrellisCoded(entry, move=True)
    assert tc.k == int(g["k"])
    tc.acc.copy_(torch.as_tensor(g["acc"]).cuda())
    new = tc.nearest(float(g["eta"]))
    assert np.array_equal(new.cpu().numpy(), g["nearest"])
    assert tc.repick(float(g["eta"])) == float(g["changed"])
    assert bool((tc.acc == 0).all())


def test_take_gradient_is_the_chain_rule():
    """take_gradient's scale and table gradients equal autograd's through matrix() (fp32, 1e-4)."""
    from lookatmyquant_b200 import codes
    from lookatmyquant_b200.finetune import TrellisCoded
    gen = torch.Generator().manual_seed(1)
    st = torch.zeros(20, 128, dtype=torch.long)
    s = torch.zeros(20, dtype=torch.long)
    for j in range(128):
        s = ((s << 2) | torch.randint(0, 4, (20,), generator=gen)) & 4095
        st[:, j] = s
    entry = {"states": st, "scales": 0.5 + torch.rand(20, generator=gen), "table": torch.randn(4096, generator=gen),
             "in_seed": 3}
    tc = TrellisCoded(entry)
    dW = torch.randn(20, 128, generator=gen).cuda()
    tc.take_gradient(dW)
    gs, gt = tc.log_s.grad.clone(), tc.table.grad.clone()
    tc.log_s.grad = tc.table.grad = None
    with torch.enable_grad():
        Q = tc.scales() * tc.table[tc.states.long()]
        W = Q @ torch.as_tensor(codes.rht(128, 3)).float().cuda()  # W = diag(S)·T[state]·R
        (W * dW).sum().backward()
    assert torch.allclose(gs, tc.log_s.grad, rtol=1e-4, atol=1e-4)
    assert torch.allclose(gt, tc.table.grad, rtol=1e-4, atol=1e-4)
