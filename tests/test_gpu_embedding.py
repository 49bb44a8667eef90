"""Embedding buckets (quantize.py:350-465) against the reference's own embed_word (tests/golden/embedding.npz): the
column trellis over runs of 256 rows after a hidden-dimension rotation, under LDLQ with H or as a lookup table
(plain Viterbi rounding, rows padded to whole runs), a centred bucket, a prng bucket. The reference rotates in fp32;
the trellis values are compared before the output rotation (Q·Rᵀ): >= 99.9 % of them equal to 1e-6, as the column
trellis's settled values are elsewhere; the stored bits exactly."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("case", ["a", "b", "c", "e"])
def test_trellis_bucket_matches_reference(golden, case):
    from lookatmyquant_b200.embedding import embed_word
    from lookatmyquant_b200.rotation import Rotation
    g = golden("embedding")
    rows, n, seed, with_h, center = (int(v) for v in g[f"{case}_meta"])
    W = torch.as_tensor(g[f"{case}_W"].astype(np.float64)).cuda()
    H = torch.as_tensor(g[f"{case}_H"].astype(np.float64)).cuda() if with_h else None
    net = embed_word(W, H, str(g[f"{case}_prog"]), seed, center=bool(center))
    Q = net.matrix().double()
    assert Q.shape == (rows, n)
    assert net.rate_bits() == float(g[f"{case}_bits"])
    R = Rotation(n, seed)
    ref = torch.as_tensor(g[f"{case}_Q"]).cuda()
    if center:  # the centred bucket adds the mean row back after the code
        m = W.mean(0, keepdim=True)
        Q, ref = Q - m, ref - m
    a, b = R.rows(Q.contiguous()), R.rows(ref.contiguous())
    close = (a - b).abs() <= 1e-6 * b.abs().max()
    assert close.double().mean() >= 0.999
    assert (Q - ref).abs().max() <= 0.5 * ref.abs().max()  # a differing state moves a row by about one table step


def test_prng_and_plain_buckets(golden):
    from lookatmyquant_b200.embedding import embed_word
    g = golden("embedding")
    W = torch.as_tensor(g["d_W"].astype(np.float64)).cuda()
    net = embed_word(W, None, "prng", 7004)
    assert torch.allclose(net.matrix(), torch.as_tensor(g["d_Q"]).cuda(), rtol=0, atol=1e-12)
    assert net.rate_bits() == float(g["d_bits"])
    assert torch.equal(embed_word(W, None, "zero", 1).matrix(), torch.zeros_like(W))
    mean = embed_word(W, None, "mean", 1).matrix()
    assert torch.allclose(mean, W.mean(0, keepdim=True).expand_as(W))


def test_quantize_embedding_writes_every_bucket():
    """A 1000-row table in three buckets (fp16, tr2 with H, zero) by frequency order: every row is written by its own
    bucket's word, the bits add up."""
    from lookatmyquant_b200.embedding import embed_word, embedding_buckets, frequency_order, quantize_embedding
    g = torch.Generator().manual_seed(0)
    E = torch.nn.Parameter((0.02 * torch.randn(1000, 64, generator=g)).to(torch.bfloat16).cuda())
    orig = E.data.clone()
    A = torch.randn(512, 64, generator=g, dtype=torch.float64)
    H = (A.T @ A / 512).cuda()
    order = frequency_order(torch.randint(0, 1000, (20000,), generator=g), 1000)
    spec = {"sizes": embedding_buckets(1000), "programs": ["fp16", "tr2", "zero"]}
    bits, numel = quantize_embedding(E, spec, H, order)
    assert numel == 1000 * 64
    r0, r1 = order[:256].cuda(), order[256:512].cuda()
    assert torch.equal(E.data[r0], orig[r0])
    want = embed_word(orig[r1].double(), H, "tr2", 7001).matrix().to(torch.bfloat16)
    assert torch.equal(E.data[r1], want)
    assert bool((E.data[order[512:].cuda()] == 0).all())
    assert bits == 16 * 256 * 64 + embed_word(orig[r1].double(), H, "tr2", 7001).rate_bits()
