"""Seeded inputs of the statistics, QEP and KL golden vectors (statistics.npz, kl.npz).

`make_golden.py` draws these inputs, runs the reference on them and stores only the outputs (and checksums of the
inputs); the tests draw the same inputs again with the same torch CPU generator and compare. A checksum mismatch
means the generator gave different numbers on this machine, and the tests say so instead of reporting a parity
failure.
"""

from __future__ import annotations

import hashlib

import torch

# (name, tokens per chunk, chunks, d, weighted): the activation streams of quantize_stage (quantize.py:1412-1470)
STAT_CASES = [("cov", 9000, 3, 96, False),   # frame.covariance: 27,000 tokens, four of its 8192-token chunks
              ("qep", 4096, 3, 128, True),   # weighted H and D, then cross_target and W·M
              ("qep_wide", 2048, 2, 256, True)]
QEP_ROWS = 64       # rows of the W whose target W·M is recorded
QEP_ALPHA = 0.5     # config 3's α

# Every input below is made from integers drawn by torch's CPU generator and combined with exactly rounded
# elementwise arithmetic (sums of integers, products with powers of two, one fp32 product and sum): no
# transcendental functions and no reductions, whose vectorised CPU kernels round differently on different CPUs.


def _gauss(shape, g: torch.Generator) -> torch.Tensor:
    """Approximately N(0, 1) fp32 values: the sum of four uniform integers in [-2048, 2048), scaled by 2^-11·√3/2."""
    u = sum(torch.randint(-2048, 2048, shape, generator=g) for _ in range(4))
    return u.to(torch.float32) * (0.8660254037844386 / 2048)


def activations(tokens: int, d: int, g: torch.Generator, scale: torch.Tensor) -> torch.Tensor:
    """bf16 activations with the given per-channel scales (powers of two)."""
    return (_gauss((tokens, d), g) * scale).to(torch.bfloat16)


def channel_scales(d: int, g: torch.Generator) -> torch.Tensor:
    """Per-channel scales 2^e, e uniform in -2..2 (a coarse lognormal), with two ×16 outlier channels."""
    e = torch.randint(-2, 3, (d,), generator=g)
    e[torch.randperm(d, generator=g)[:2]] += 4
    return torch.tensor([2.0 ** int(v) for v in e], dtype=torch.float32)


def stat_inputs(name: str):
    """(xq chunks, xr chunks or None, token-weight chunks or None, W or None): bf16 chunks on the CPU."""
    case = next(c for c in STAT_CASES if c[0] == name)
    _, tokens, nchunks, d, weighted = case
    g = torch.Generator().manual_seed(7000 + tokens + d)
    scale = channel_scales(d, g)
    gain = 1.0 + torch.randint(-100, 101, (d,), generator=g).to(torch.float32) / 1024 if weighted else None
    xq, xr, w = [], [], []
    for _ in range(nchunks):
        x = activations(tokens, d, g, scale)
        xq.append(x)
        if weighted:  # the reference stream: the quantized one with per-channel gains of ±10 % and some noise
            xr.append((x.float() * gain + 0.0625 * _gauss((tokens, d), g)).to(torch.bfloat16))
            w.append(torch.where(torch.randint(0, 100, (tokens,), generator=g) < 8, 10.0, 1.0).float())
    W = (_gauss((QEP_ROWS, d), g).double() * (1.0 / 64)) if weighted else None
    return xq, (xr if weighted else None), (w if weighted else None), W


def kl_inputs():
    """A tiny random-init Llama (bf16; weights N(0, 0.3²) so the logits spread over a few nats), its 'probe' copy with one linear piece perturbed, and held token ids."""
    from transformers import LlamaConfig, LlamaForCausalLM
    cfg = LlamaConfig(hidden_size=64, intermediate_size=128, num_hidden_layers=2, num_attention_heads=4,
                      num_key_value_heads=2, vocab_size=1000, rms_norm_eps=1e-5, rope_theta=1e4,
                      tie_word_embeddings=True, max_position_embeddings=256, initializer_range=0.3)
    cfg._attn_implementation = "eager"
    torch.manual_seed(31)
    ref = LlamaForCausalLM(cfg).to(torch.bfloat16).eval()
    probe = LlamaForCausalLM(cfg).to(torch.bfloat16).eval()
    probe.load_state_dict(ref.state_dict())
    g = torch.Generator().manual_seed(32)
    with torch.no_grad():
        w = probe.model.layers[1].mlp.down_proj.weight
        w.copy_((w.float() + 0.2 * torch.randn(w.shape, generator=g)).to(torch.bfloat16))
    ranks = torch.arange(1, cfg.vocab_size + 1, dtype=torch.float64).pow(-1.1)
    ids = torch.multinomial(ranks, 3 * 96, replacement=True, generator=g).reshape(3, 96)
    return ref, probe, ids


def digest(tensors) -> str:
    """SHA-256 of the tensors' bytes, in order."""
    h = hashlib.sha256()
    for t in tensors:
        h.update(t.contiguous().view(torch.uint8).numpy().tobytes() if t.dtype == torch.bfloat16
                 else t.contiguous().numpy().tobytes())
    return h.hexdigest()


def tiny_llama(dtype=None, state=None):
    """A 2-layer Llama of hidden 64 (vocab 1000, weights N(0, 0.3²) rounded to bf16 values), fp32 unless `dtype`;
    `state` loads given weights (the fixture's) instead of the seeded initialisation."""
    from transformers import LlamaConfig, LlamaForCausalLM
    cfg = LlamaConfig(hidden_size=64, intermediate_size=128, num_hidden_layers=2, num_attention_heads=4,
                      num_key_value_heads=2, vocab_size=1000, rms_norm_eps=1e-5, rope_theta=1e4,
                      tie_word_embeddings=True, max_position_embeddings=256, initializer_range=0.3)
    cfg._attn_implementation = "eager"
    torch.manual_seed(41)
    model = LlamaForCausalLM(cfg).eval()
    if state is not None:
        model.load_state_dict(state)
    else:
        with torch.no_grad():
            for p in model.parameters():
                p.copy_(p.to(torch.bfloat16).float())
    return model.to(dtype or torch.float32)
