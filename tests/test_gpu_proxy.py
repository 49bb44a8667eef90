"""The proxy loss on the device (lamq_proxy_loss) and best_word's seed selection (quantize.py:1316-1328).

The proxy loss is the reference's (E @ H * E).sum() with E = word − target, in fp64: against numpy's fp64 to 1e-12
relative. best_word is checked against the reference's own best_word (tests/golden/best_word.npz): the same seed is
chosen, each candidate's error within the 0.5 % proxy-loss bar, and the chosen word's states."""

import numpy as np
import pytest
import torch


pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rows,n,with_target", [(64, 128, True), (5000, 256, True), (77, 320, False), (1, 16, True)])
def test_proxy_loss_matches_fp64(rows, n, with_target):
    from lookatmyquant_b200.frame import proxy_loss
    rng = np.random.default_rng(rows + n)
    A = rng.standard_normal((2 * n, n))
    H = A.T @ A / (2 * n)
    Wq = 0.02 * rng.standard_normal((rows, n))
    W = Wq + 0.001 * rng.standard_normal((rows, n)) if with_target else None
    E = Wq - W if with_target else Wq
    want_rows = ((E @ H) * E).sum(1)
    total, per_row = proxy_loss(torch.as_tensor(Wq).cuda(), None if W is None else torch.as_tensor(W).cuda(),
                                torch.as_tensor(H).cuda(), per_row=True)
    assert abs(float(total) - want_rows.sum()) <= 1e-12 * abs(want_rows.sum())
    assert np.abs(per_row.cpu().numpy() - want_rows).max() <= 1e-12 * np.abs(want_rows).max()
    again = proxy_loss(torch.as_tensor(Wq).cuda(), None if W is None else torch.as_tensor(W).cuda(),
                       torch.as_tensor(H).cuda())
    assert float(again) == float(total)  # fixed summation order


def test_proxy_loss_of_a_strided_word():
    """Non-contiguous rows (a slice of a wider matrix) are read through their leading dimension."""
    from lookatmyquant_b200.frame import proxy_loss
    rng = np.random.default_rng(3)
    H = np.eye(64) + 0.1
    big = torch.as_tensor(rng.standard_normal((40, 100))).cuda()
    Wq = big[:, 10:74]
    want = float(((Wq.cpu().numpy() @ H) * Wq.cpu().numpy()).sum())
    got = float(proxy_loss(Wq, None, torch.as_tensor(H).cuda()))
    assert abs(got - want) <= 1e-12 * abs(want)


def test_best_word_matches_reference(golden):
    from lookatmyquant_b200 import codes, quantize
    g = golden("best_word")
    m, n, k, seed, nseeds = (int(v) for v in g["meta"])
    W = torch.as_tensor(g["W"].astype(np.float64)).cuda()
    H = torch.as_tensor(g["H"].astype(np.float64)).cuda()
    trellis = {b: codes.RowTrellisCode(12, b, T=256, width=16, look=8) for b in (1, 2, 3, 4)}
    net, errs = quantize.best_word(f"tr{k}", W, H, seed, trellis, seeds=nseeds)
    errs = errs.cpu().numpy()
    assert np.all(np.abs(errs - g["errs"]) <= 0.005 * g["errs"])
    assert int(np.argmin(errs)) == int(g["chosen"])
    st = net.states.cpu().numpy().astype(np.int64)
    assert (st == g["states"]).mean() >= 0.999
    # a single seed: the plain word, no errors
    one, none = quantize.best_word(f"tr{k}", W, H, seed, trellis, seeds=1)
    assert none is None and torch.equal(one.states, codes.ldlq_words([W], H, trellis[k], [seed])[0].states)


def test_environment_error_is_the_proxy_loss():
    from lookatmyquant_b200.frame import Environment
    rng = np.random.default_rng(5)
    A = rng.standard_normal((300, 96))
    H = torch.as_tensor(A.T @ A / 300).cuda()
    env = Environment(H)
    D = torch.as_tensor(0.01 * rng.standard_normal((20, 96))).cuda()
    Hd = env.H.cpu().numpy()
    want = float(np.trace(D.cpu().numpy() @ Hd @ D.cpu().numpy().T))
    assert abs(env.error(D) - want) <= 1e-12 * abs(want)
