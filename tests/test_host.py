"""Host logic that needs no GPU: table lookup and caching, the generic sweep's steps on host tensors."""

import numpy as np
import pytest
import torch


def test_missing_table_is_fitted_and_cached(tmp_path, monkeypatch):
    from lookatmyquant_b200 import codes
    monkeypatch.setattr(codes, "fit_trellis_values", lambda *a, **kw: torch.arange(4096.0))
    monkeypatch.setenv("LAMQ_TABLE_CACHE", str(tmp_path))
    v = codes.trellis_values(12, 2, 48)
    assert (tmp_path / "trellis_L12_k2_T48_s0_ema.f64").exists()
    assert np.array_equal(codes.trellis_values(12, 2, 48).numpy(), v.numpy())


def test_zipf_tokens_are_seeded_and_in_range():
    from lookatmyquant_b200 import measure
    a = measure.zipf_tokens(3, 50, 1000, 7)
    b = measure.zipf_tokens(3, 50, 1000, 7)
    assert torch.equal(a, b) and a.shape == (3, 50) and int(a.min()) >= 0 and int(a.max()) < 1000
    assert (a == 0).float().mean() > (a == 10).float().mean()  # rank 1 is the most frequent


def test_smollm2_shape():
    from lookatmyquant_b200 import measure
    c = measure.smollm2_config()
    assert (c.hidden_size, c.intermediate_size, c.num_hidden_layers, c.num_attention_heads, c.num_key_value_heads,
            c.vocab_size, c.tie_word_embeddings) == (960, 2560, 32, 15, 5, 49152, True)


def test_shipped_tables_match_their_sums():
    import hashlib
    from lookatmyquant_b200 import codes
    lines = (codes.TABLES / "SHA256SUMS").read_text().split("\n")
    sums = dict(reversed(line.split("  ")) for line in lines if line)
    assert len(sums) == 7
    for name, h in sums.items():
        assert hashlib.sha256((codes.TABLES / name).read_bytes()).hexdigest() == h
        assert np.fromfile(codes.TABLES / name, dtype="<f8").shape == (4096,)


class _Env:
    """The two attributes the sweep reads from an environment."""

    def __init__(self, U, dead):
        self.U, self.dead = U, dead


@pytest.mark.parametrize("width", [1, 4])
def test_generic_sweep_matches_reference_on_cpu(golden, width):
    """syntax.sweep (syntax.py:86-124) with a Python nearest-level projection, on the host, against the reference's
    own sweep of the same inputs (the environment's U from the oracle, itself pinned to the reference's)."""
    from lookatmyquant_b200 import syntax
    from oracle import core as O
    g = golden("ldlq_gpu")
    Hd = g["H"].copy()
    Hd[5, :] = 0
    Hd[:, 5] = 0
    U, dead, _ = O.environment(Hd)
    lv = torch.as_tensor(g["levels8"])
    mids = (lv[1:] + lv[:-1]) / 2

    def nearest(j, cols, T):
        return lv[torch.bucketize(cols.contiguous(), mids)]
    got = syntax.sweep(torch.as_tensor(g["X"]), _Env(torch.as_tensor(U), torch.as_tensor(dead)), nearest, width=width,
                       lazy=64).numpy()
    ref = g[f"sweep_w{width}"]
    assert np.abs(got - ref).max() <= 1e-10 * np.abs(ref).max()


def test_program_names_parse_like_reference():
    from lookatmyquant_b200.quantize import Dense, parse, word
    assert parse("tr2") == ("tr", 2, False) and parse("tr3x") == ("tr", 3, True)
    assert parse("fp16") == ("fp", 16, False) and parse("gptaq4") == ("gptaq", 4, True)
    for bad in ("tr", "rtn2x", "q4", "orig"):
        with pytest.raises(ValueError, match="unknown program"):
            parse(bad)
    W = torch.randn(4, 8, dtype=torch.float64)
    d = word("fp16", W, None, 0, {})
    assert isinstance(d, Dense) and d.rate_bits() == 16 * 32
    assert torch.equal(d.matrix(), W.to(torch.bfloat16).double())
    with pytest.raises(NotImplementedError):
        word("rtn4", W, None, 0, {})


def test_generic_sweep_without_environment_returns_the_columns():
    """With no environment there is no Refit: the columns as they stood are W's, and the projection sees each one."""
    from lookatmyquant_b200 import syntax
    W = torch.randn(5, 12, dtype=torch.float64)
    seen = []

    def project(j, cols, T):
        seen.append(j)
        return cols.round()
    out = syntax.sweep(W, None, project, width=3, lazy=6)
    assert torch.equal(out, W) and seen == [0, 3, 6, 9]


def test_scalar_ldlq_rejects_blocks_over_128():
    from lookatmyquant_b200.ldlq_gpu import ldlq_round
    with pytest.raises(ValueError, match="block"):
        ldlq_round(torch.zeros(2, 4), torch.eye(4), torch.tensor([0.0, 1.0]), block=256)


@pytest.mark.parametrize("width", [1, 4])
def test_generic_sweep_refit_is_least_squares(width):
    """As the reference's test_frame.py:51-62 and test_codes.py:64-75: just before a block is settled, the sweep's
    running values of the unsettled columns are the least-squares best continuation of the settled ones,
    X_r = W_r + (W_s − Q_s)·H_sr·H_rr⁻¹, with H the damped statistics whose inverse the environment's U factors."""
    from lookatmyquant_b200 import syntax
    from oracle import core as O
    rng = np.random.default_rng(3)
    n, rows = 16, 5
    A = rng.standard_normal((64, n))
    U, dead, Hd = O.environment(A.T @ A / 64)
    W = rng.standard_normal((rows, n))
    settled = np.zeros((rows, n))

    def quarter(j, cols, T):
        q = torch.round(cols * 4) / 4
        settled[:, j:j + width] = q.reshape(rows, width).numpy()
        return q
    before = syntax.sweep(torch.as_tensor(W), _Env(torch.as_tensor(U), torch.as_tensor(dead)), quarter, width=width,
                          lazy=8).numpy()
    for j in range(0, n, width):
        s, r = slice(0, j), slice(j, n)
        best = W[:, r] + (W[:, s] - settled[:, s]) @ Hd[s, r] @ np.linalg.inv(Hd[r, r])
        assert np.abs(before[:, j:j + width] - best[:, :width]).max() < 1e-10


def test_generic_sweep_rows_do_not_interact():
    """As the reference's test_codes.py:87-99: under Refit the rows are independent, so sweeping a stacked matrix
    equals sweeping its halves apart — the property that lets the rows of a stage be split across GPUs."""
    from lookatmyquant_b200 import syntax
    from oracle import core as O
    rng = np.random.default_rng(4)
    n = 24
    A = rng.standard_normal((96, n))
    U, dead, _ = O.environment(A.T @ A / 96)
    env = _Env(torch.as_tensor(U), torch.as_tensor(dead))
    W = torch.as_tensor(rng.standard_normal((7, n)))

    def half(j, cols, T):
        return torch.round(cols * 2) / 2
    whole = syntax.sweep(W, env, half, width=4, lazy=8)
    parts = torch.cat([syntax.sweep(W[:3], env, half, width=4, lazy=8), syntax.sweep(W[3:], env, half, width=4,
                                                                                       lazy=8)])
    assert torch.allclose(whole, parts, rtol=0, atol=1e-12)


def test_shipped_two_bit_trellis_beats_scalar_on_gaussians():
    """As the reference's test_codes.py:134-144 (2 bits per weight on unit Gaussians: the 4-level Lloyd-Max scalar
    quantizer has distortion ≈ 0.1175, a trellis code beats it by more than 0.01), for the shipped 4096-state k = 2
    table that the B200 sweep uses, decoded by the oracle's Viterbi (the GPU decoder's states equal it bit for bit)."""
    from lookatmyquant_b200 import codes
    from oracle import core as O
    X = np.random.default_rng(5).standard_normal((48, 256))
    levels = np.array([-1.510, -0.4528, 0.4528, 1.510])  # the Lloyd-Max quantizer of N(0, 1) at 2 bits
    scalar = np.mean(np.min((X[..., None] - levels) ** 2, axis=-1))
    assert abs(scalar - 0.1175) < 0.005
    values = codes.trellis_values(12, 2, 256).numpy()
    states = O.viterbi(X, values, 12, 2)
    assert O.is_trellis_path(states, 12, 2)
    trellis = np.mean((X - values.astype(np.float32)[states]) ** 2)
    assert trellis < scalar - 0.01


def test_column_trellis_layout_and_price():
    """As the reference's test_codes.py:120-131: a column trellis cuts each column into sequences of T consecutive
    outputs (its W.reshape(o/T, T, w).permute(0, 2, 1) layout), and a word whose sequences start anywhere pays L − k
    bits per sequence on top of k per entry (plus 16 per row scale and one sign per rotated input, as our words
    carry both)."""
    from lookatmyquant_b200 import codes
    code = codes.TrellisCode(12, 2, 256)
    W = torch.randn(512, 8, dtype=torch.float64)
    assert torch.equal(code._seqs(W), W.reshape(2, 256, 8).permute(0, 2, 1).reshape(-1, 256))
    m, n, T = 512, 8, 256
    word = codes.TrellisWord(torch.zeros(m, n, dtype=torch.int16), torch.ones(m), torch.zeros(m, n), code.values, 12,
                             2, None, None, fixed_start=False, T=T)
    assert word.rate_bits() == m * n * 2 + 16 * m + (m * n // T) * (12 - 2)
    word.fixed_start = True
    assert word.rate_bits() == m * n * 2 + 16 * m


def test_cpu_baseline_fit_separates_call_and_row_costs(monkeypatch):
    """The CPU baseline's word timing: a line through two sample sizes gives the cost per call and per row, so a
    small sample's fixed cost is not multiplied by the layer's rows; times out of order fall back to the larger
    sample's time per row."""
    import bench
    times = {16: 1.0 + 16 * 0.01, 128: 1.0 + 128 * 0.01}
    monkeypatch.setattr(bench, "_words_seconds", lambda W, *a: times[W.shape[0]])
    per_call, per_row = bench.words_fit(np.zeros((128, 8)), None, None, None, None)
    assert abs(per_call - 1.0) < 1e-9 and abs(per_row - 0.01) < 1e-12
    times[128] = 0.9  # noise: the larger sample ran faster
    assert bench.words_fit(np.zeros((128, 8)), None, None, None, None) == (0.0, 0.9 / 128)


def test_embedding_buckets_and_frequency_order_match_reference(golden):
    """quantize.py:350-364 by the reference (embedding.npz): bucket sizes and the frequency order (ties by id)."""
    import torch
    from lookatmyquant_b200.embedding import embedding_buckets, frequency_order
    g = golden("embedding")
    assert embedding_buckets(49152) == list(g["buckets_49152"])
    assert embedding_buckets(1000) == list(g["buckets_1000"])
    assert torch.equal(frequency_order(torch.as_tensor(g["freq_ids"]), 600), torch.as_tensor(g["freq_order"]))


def test_synthetic_codebooks_match_reference(golden):
    """BASELINE config 3's codebooks: nested.lloyd_max_levels restated (fp64, to 1e-12), and the fp16 levels in
    the state order trellis_values gives its quantiles, exactly (small_l.npz, by the reference)."""
    import torch
    from lookatmyquant_b200.codes import lloyd_max_levels, synthetic_codebook
    g = golden("small_l")
    assert np.abs(lloyd_max_levels(64).numpy() - g["lloyd_max_levels_64"]).max() <= 1e-12
    for bits in (1, 2, 3, 4):
        L, v = synthetic_codebook(bits)
        assert L == bits + 4 and torch.equal(v, torch.as_tensor(g[f"codebook_{bits}"]))


@pytest.mark.parametrize("n", [2560, 4096, 9728, 960, 1536])
def test_hadamard_factor_a_is_the_sylvester_pattern_the_device_checks(n):
    """Every A of hadamard_factors (and B when it is a power-of-two Sylvester matrix) has exactly the sign bits the
    rotation kernel's device check accepts for its butterfly path: bit k of word w of row r set iff
    popcount(r & (32w + k)) is odd."""
    from lookatmyquant_b200.codes import hadamard_factors
    from lookatmyquant_b200.rotation import _sign_bits
    A, B = hadamard_factors(n)

    def pattern(order):
        words = (order + 31) // 32
        out = np.zeros((order, words), dtype=np.uint32)
        for r in range(order):
            for c in range(order):
                if bin(r & c).count("1") & 1:
                    out[r, c // 32] |= np.uint32(1) << np.uint32(c % 32)
        return out

    a = A.shape[0]
    assert a & (a - 1) == 0
    assert np.array_equal(_sign_bits(A).numpy().view(np.uint32), pattern(a))
    b = B.shape[0]
    if b & (b - 1) == 0 and b > 2:
        assert np.array_equal(_sign_bits(B).numpy().view(np.uint32), pattern(b))


def test_host_build_takes_the_stage_with_the_least_work_last():
    """build_layer_from_host copies and builds the stages in order of the work after their statistics (the largest
    factorization and sweep first), the same order on every rank."""
    from lookatmyquant_b200.layer import qwen3_4b_stages, tail_order
    stages = qwen3_4b_stages()
    one = [s.name for s in tail_order(stages, 1)]
    assert one[0] == "down_in" and one[-1] == "o_in"
    assert [s.name for s in tail_order(list(reversed(stages)), 1)] == one
    eight = [s.name for s in tail_order(stages, 8)]
    assert eight[0] == "down_in" and set(eight) == set(one)
