"""The drop-in boundary at the reference's own call sites (tests/golden/dropin.npz): the reference's
quantize_row_groups (quantize.py:530-565) ran with every call to opgraph.codes.ldlq_words and opgraph.codes.viterbi
recorded. Each recorded call is replayed into this package's function of the same name and signature
(lookatmyquant_b200.codes.viterbi, .ldlq_words with RowTrellisCode): identical results at every call means the
reference, with these two names bound to the package, takes the same path call for call."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_every_recorded_viterbi_call_replays_identically(golden):
    from lookatmyquant_b200 import codes
    g = golden("dropin")
    off_x = off_s = 0
    for k, rows, T in zip(g["vit_k"], g["vit_rows"], g["vit_T"]):
        X = torch.as_tensor(g["vit_X"][off_x:off_x + rows * T].reshape(rows, T))
        start = torch.as_tensor(g["vit_start"][off_s:off_s + rows])
        want = g["vit_out"][off_x:off_x + rows * T].reshape(rows, T)
        got = codes.viterbi(X, codes.trellis_values(12, int(k), 256), 12, int(k), start=start)
        assert np.array_equal(got.cpu().numpy(), want)
        off_x += rows * T
        off_s += rows
    assert off_x == len(g["vit_X"])


def test_every_recorded_ldlq_words_call_replays_identically(golden):
    from lookatmyquant_b200 import codes
    g = golden("dropin")
    H = torch.as_tensor(g["H"].astype(np.float64))
    for i in range(int(g["words_calls"])):
        k, seed, inc, in_seed, out_rot = (int(v) for v in g[f"w{i}_meta"])
        W = torch.as_tensor(g[f"w{i}_W"].astype(np.float64))
        code = codes.RowTrellisCode(12, k, T=256, width=16, look=8)
        word = codes.ldlq_words([W], H, code, [seed], incoherent=bool(inc), in_seed=None if in_seed < 0 else in_seed,
                                out_rot=bool(out_rot))[0]
        assert np.array_equal(word.states.cpu().numpy().astype(np.int64), g[f"w{i}_states"])
