"""The column-trellis sweep (TrellisCode, opgraph/codes.py:363-383: the `measure` path's trellis words, two-sided
rotation) on the GPU, against the reference's own ldlq_words output (tests/golden/column_trellis.npz) and the oracle's
column_trellis_sweep; and the words without H (the code applied directly, codes.py:460-461)."""

import numpy as np
import pytest
import torch

import oracle.core as O
from conftest import table

pytestmark = pytest.mark.gpu


def test_column_trellis_word_matches_reference(golden):
    from lookatmyquant_b200 import codes
    g = golden("column_trellis")
    m, n, k, seed, Tm = (int(x) for x in g["meta"])
    code = codes.TrellisCode(12, k, T=Tm)
    word = codes.ldlq_words([torch.as_tensor(g["W"].astype(np.float64))], torch.as_tensor(g["H"].astype(np.float64)),
                            code, [seed])[0]
    settled = word.settled.cpu().numpy()
    assert (settled == g["settled"]).mean() >= 0.999
    assert np.abs(word.scales.cpu().numpy() - g["S"]).max() < 1e-12
    Wq = word.matrix().cpu().numpy()
    assert np.abs(Wq - g["Wq"]).max() <= 1e-3 * np.abs(g["Wq"]).max()


@pytest.mark.parametrize("k,Tm,m,n", [(1, 64, 192, 96), (3, 128, 256, 160), (4, 32, 96, 80), (2, 256, 512, 136)])
def test_column_sweep_matches_oracle(k, Tm, m, n):
    """The sweep kernel alone against the oracle: ragged runs of the lazy window (n not a multiple of 128) and a
    partial last block (n not a multiple of 16)."""
    from lookatmyquant_b200 import codes
    from lookatmyquant_b200.frame import Environment
    rng = np.random.default_rng(k * 1000 + n)
    A = rng.standard_normal((2 * n, n)) * np.exp(rng.standard_normal(n))
    H = A.T @ A / (2 * n)
    H[7, :] = 0
    H[:, 7] = 0  # a dead input
    X = 0.02 * rng.standard_normal((m, n))
    S = O.row_scale(X)
    U, dead, _ = O.environment(H)
    before_o, settled_o, states_o = O.column_trellis_sweep(X, S, U, dead, table(k), 12, k, Tm)
    env = Environment(torch.as_tensor(H).cuda())
    code = codes.TrellisCode(12, k, T=256)
    code.T = Tm  # runs of Tm rows with the shipped T = 256 table
    before, states, settled = codes._col_trellis_sweep(torch.as_tensor(X).cuda(), torch.as_tensor(S).cuda(), env, code)
    st = states.cpu().numpy().astype(np.int64)
    assert (st == states_o).mean() >= 0.999
    if (st == states_o).all():
        assert np.abs(before.cpu().numpy() - before_o).max() <= 1e-12 * np.abs(before_o).max()


@pytest.mark.parametrize("kind", ["row", "column"])
def test_words_without_H_round_to_the_nearest_path(kind):
    from lookatmyquant_b200 import codes
    rng = np.random.default_rng(5)
    W = torch.as_tensor(0.02 * rng.standard_normal((128, 64)))
    code = codes.RowTrellisCode(12, 2) if kind == "row" else codes.TrellisCode(12, 2, T=256)
    code.T = 64 if kind == "column" else code.T
    word = codes.ldlq_words([W], None, code, [3], out_rot=(kind == "column"))[0]
    X = word.R_in.rows(W.cuda())
    if word.R_out is not None:
        X = word.R_out.rows(X.T.contiguous()).T.contiguous()
    xs = (X / word.scales[:, None]).cpu().numpy()
    if kind == "row":
        ref = O.viterbi(xs, table(2), 12, 2, start=np.zeros(len(xs), dtype=np.int64))
    else:
        seqs = xs.reshape(2, 64, 64).transpose(0, 2, 1).reshape(-1, 64)
        ref = O.viterbi(seqs, table(2), 12, 2).reshape(2, 64, 64).transpose(0, 2, 1).reshape(128, 64)
    assert np.array_equal(word.states.cpu().numpy().astype(np.int64), ref)
