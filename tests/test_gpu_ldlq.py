"""GPU parity: the fused row-trellis LDLQ sweep (lamq_ldlq_rowtrellis) and ldlq_words against the reference's golden
words and the oracle. Bars (north star): >= 99.9% identical code indices, proxy loss within 0.5%."""

import numpy as np
import pytest
import torch

from conftest import table
from oracle import core as O

pytestmark = pytest.mark.gpu


def kernel_sweep(X, S, U, dead, k, row_bits=None, width=16, look=8):
    from lookatmyquant_b200 import _lib
    from lookatmyquant_b200.codes import stacked_tables
    dev = torch.device("cuda")
    T = torch.as_tensor(np.ascontiguousarray(X, dtype=np.float64)).to(dev)
    rows, n = T.shape
    Ut = torch.as_tensor(np.ascontiguousarray(U, dtype=np.float64)).to(dev)
    St = torch.as_tensor(np.asarray(S, dtype=np.float64)).to(dev)
    dd = None if dead is None or not np.any(dead) else torch.as_tensor(np.asarray(dead, dtype=np.uint8)).to(dev)
    rb = None if row_bits is None else torch.as_tensor(np.asarray(row_bits, dtype=np.uint8)).to(dev)
    tabs = stacked_tables(12, 256, dev)
    states = torch.empty(rows, n, dtype=torch.int16, device=dev)
    settled = torch.empty(rows, n, dtype=torch.float64, device=dev)
    ws = torch.empty(_lib.load().lamq_ldlq_rowtrellis_workspace_size(rows, n), dtype=torch.uint8, device=dev)
    _lib.check(_lib.load().lamq_ldlq_rowtrellis(
        T.data_ptr(), n, rows, n, Ut.data_ptr(), n, None if dd is None else dd.data_ptr(), St.data_ptr(),
        tabs.data_ptr(), None if rb is None else rb.data_ptr(), k, 12, width, look, 128, states.data_ptr(),
        settled.data_ptr(), ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream), "sweep")
    torch.cuda.synchronize()
    return T.cpu().numpy(), states.cpu().numpy().astype(np.int64), settled.cpu().numpy()


@pytest.mark.parametrize("case", ["a", "b", "c", "d"])
def test_kernel_matches_oracle_sweep(golden, case):
    """Same X, S and U in: the kernel's states equal the oracle's (and so the reference's) exactly."""
    g = golden("ldlq_row")
    m, n, k, seed, in_seed = (int(x) for x in g[f"{case}_meta"])
    W, H = g[f"{case}_W"].astype(np.float64), g[f"{case}_H"].astype(np.float64)
    R = O.rht(n, in_seed)
    X = W @ R.T
    S = O.row_scale(X)
    U, dead, _ = O.environment(R @ H @ R.T)
    before_o, settled_o, states_o = O.row_trellis_sweep(X, S, U, dead, table(k), 12, k)
    before, states, settled = kernel_sweep(X, S, U, dead, k)
    assert np.array_equal(states, g[f"{case}_states"].astype(np.int64))
    assert np.array_equal(states, states_o)
    assert np.array_equal(settled, settled_o)
    assert np.abs(before - before_o).max() <= 1e-12 * np.abs(before_o).max()


def test_kernel_dead_inputs_no_rotation(golden):
    g = golden("ldlq_row")
    m, n, k = (int(x) for x in g["e_meta"][:3])
    W, H = g["e_W"].astype(np.float64), g["e_H"].astype(np.float64)
    S = O.row_scale(W)
    U, dead, _ = O.environment(H)
    _, states, settled = kernel_sweep(W, S, U, dead, k)
    assert np.array_equal(states, g["e_states"].astype(np.int64))


def test_kernel_mixed_row_widths(golden):
    """A row plan: each row its own k (one kernel for all groups; rows do not interact)."""
    g = golden("row_groups")
    W, H, perm = g["W"].astype(np.float64), g["H"].astype(np.float64), g["perm"]
    n = W.shape[1]
    in_seed = int(g["in_seed"])
    R = O.rht(n, in_seed)
    X = W @ R.T
    S = O.row_scale(X)
    U, dead, _ = O.environment(R @ H @ R.T)
    bits = np.empty(len(W), dtype=np.int64)
    table_index = np.empty(len(W), dtype=np.int64)
    for ti, b in enumerate(g["bits"]):
        bits[perm[ti * 64:(ti + 1) * 64]] = b
        table_index[perm[ti * 64:(ti + 1) * 64]] = ti
    _, states, _ = kernel_sweep(X, S, U, dead, 0, row_bits=bits)
    assert np.array_equal(states + 4096 * table_index[:, None], g["states"].astype(np.int64))


@pytest.mark.parametrize("width,look", [(16, 8), (8, 4), (16, 0), (4, 12), (8, 16)])
def test_kernel_other_windows(width, look):
    rng = np.random.default_rng(width * 100 + look)
    m, n, k = 40, 192, 2
    A = rng.standard_normal((512, n)) * np.exp(rng.standard_normal(n))
    H = A.T @ A / 512
    X = 0.02 * rng.standard_normal((m, n))
    S = O.row_scale(X)
    U, dead, _ = O.environment(H)
    _, _, st_o = O.row_trellis_sweep(X, S, U, dead, table(k), 12, k, width=width, look=look)
    _, st, _ = kernel_sweep(X, S, U, dead, k, width=width, look=look)
    assert (st == st_o).mean() >= 0.999


@pytest.mark.parametrize("case", ["a", "b", "c", "d"])
def test_ldlq_words_match_reference(golden, case):
    """The whole word on the GPU (rotation, scales, environment, sweep, dequantization) against the reference."""
    from lookatmyquant_b200 import codes
    g = golden("ldlq_row")
    m, n, k, seed, in_seed = (int(x) for x in g[f"{case}_meta"])
    W = torch.as_tensor(g[f"{case}_W"].astype(np.float64))
    H = torch.as_tensor(g[f"{case}_H"].astype(np.float64))
    code = codes.RowTrellisCode(12, k, T=256, width=16, look=8)
    word = codes.ldlq_words([W], H.cuda(), code, [seed], in_seed=in_seed, out_rot=False)[0]
    states = word.states.cpu().numpy().astype(np.int64)
    assert (states == g[f"{case}_states"]).mean() >= 0.999
    Wq = word.matrix().cpu().numpy()
    E = Wq - W.numpy()
    proxy = float(np.sum((E @ H.numpy()) * E))
    assert abs(proxy - float(g[f"{case}_proxy"])) <= 0.005 * float(g[f"{case}_proxy"])
    assert np.abs(word.scales.cpu().numpy() - g[f"{case}_S"]).max() < 1e-12
    assert word.rate_bits() == m * n * k + 16 * m + n


def test_config1_shape_against_oracle():
    """Config-1 shape (2560 x 960, k = 2, the gate_proj seeds of layer 0): states and proxy loss against the oracle."""
    from lookatmyquant_b200 import codes
    from lookatmyquant_b200.workloads import config1
    W, H, seed, in_seed = config1()
    ref = O.ldlq_row_words(W.numpy(), H.numpy(), table(2), 12, 2, in_seed)
    code = codes.RowTrellisCode(12, 2, T=256, width=16, look=8)
    word = codes.ldlq_words([W], H.cuda(), code, [seed], in_seed=in_seed, out_rot=False)[0]
    st = word.states.cpu().numpy().astype(np.int64)
    assert (st == ref["states"]).mean() >= 0.999
    Wq = word.matrix().cpu().numpy()
    E = Wq - W.numpy()
    proxy = float(np.sum((E @ H.numpy()) * E))
    assert abs(proxy - ref["proxy"]) <= 0.005 * ref["proxy"]


def test_word_cores_give_the_states_as_the_reference_saves_them():
    """quantize.word for a trellis program returns a Net-like word whose cores are what quantize.py reads to save codes
    (trellis_code_entry, quantize.py:513-527): the states recovered from cores["W"] by table lookup are the word's."""
    from lookatmyquant_b200 import codes
    from lookatmyquant_b200.quantize import word
    g = torch.Generator().manual_seed(2)
    W = 0.02 * torch.randn(64, 256, generator=g, dtype=torch.float64)
    A = torch.randn(1024, 256, generator=g, dtype=torch.float64)
    H = A.T @ A / 1024
    w = word("tr2", W.cuda(), H.cuda(), 7, {2: codes.RowTrellisCode(12, 2)}, in_seed=301, out_rot=False)
    core = w.cores["W"]
    table = torch.as_tensor(core.domain.levels, dtype=torch.float64)
    assert len(table) == 4096 and core.domain.fixed_start and "I[u]" not in w.cores
    v = core.data.double().cpu()
    st, order = table.sort()
    pos = torch.searchsorted(st, v.contiguous()).clamp(1, len(st) - 1)
    pos = torch.where((v - st[pos - 1]).abs() <= (st[pos] - v).abs(), pos - 1, pos)
    # tables can hold equal values; compare the values the states stand for
    assert torch.equal(table[order[pos]], table[w.states.long().cpu()])
    assert w.cores["W.S"].data.flatten().shape == (64,)
    assert w.matrix().shape == W.shape and w.rate_bits() > 0
