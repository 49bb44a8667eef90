"""Seeded synthetic inputs with the shapes and distributions of the benchmark configurations.

No public dataset or checkpoint is involved: every configuration is synthetic (weights N(0, 0.02²), activations
Gaussian with lognormal per-channel scales). Generators use torch's CPU generator so every machine draws the same
numbers. Seeds follow quantize.py:1492-1493: seed = 1000·layer + 100·block_seed + j, in_seed = 1000·layer +
100·block_seed(first) + 1, with block_seed("mlp") = 3, block_seed("self_attn") = 2 (compiler_arch.py:75-77).
"""

from __future__ import annotations

import torch

BLOCK_SEED = {"self_attn": 2, "mlp": 3}


def seeds_for(layer: int, name: str, j: int, first: str | None = None) -> tuple[int, int]:
    """(seed, in_seed) of matrix `name`, j-th in its stage (quantize.py:1492-1493, --rot in-shared)."""
    head = name.split(".")[0]
    seed = 1000 * layer + 100 * BLOCK_SEED[head] + j
    in_seed = 1000 * layer + 100 * BLOCK_SEED[(first or name).split(".")[0]] + 1
    return seed, in_seed


def calibration(tokens: int, d: int, seed: int, outliers: int = 4, dtype=torch.float32) -> torch.Tensor:
    """Gaussian tokens with per-channel std lognormal(0, 1); `outliers` fixed channels scaled ×20."""
    g = torch.Generator().manual_seed(seed)
    std = torch.exp(torch.randn(d, generator=g))
    if outliers:
        std[torch.randperm(d, generator=g)[:outliers]] *= 20
    return (torch.randn(tokens, d, generator=g) * std).to(dtype)


def config1():
    """Config 1: SmolLM2-360M gate_proj [2560 × 960] fp32 ~ N(0, 0.02²) from seed 0; X 16,384 × 960 fp32 with
    lognormal channel scales and 4 outlier channels ×20; H = XᵀX / 16,384 (fp64). Seeds of layer 0 mlp.gate_proj.
    Returns (W fp64, H fp64, seed, in_seed), on the CPU."""
    g = torch.Generator().manual_seed(0)
    W = (0.02 * torch.randn(2560, 960, generator=g)).double()
    X = calibration(16384, 960, seed=1).double()
    H = X.T @ X / 16384
    seed, in_seed = seeds_for(0, "mlp.gate_proj", 0)
    return W, H, seed, in_seed


def activations_bf16(tokens: int, d: int, seed: int, device="cuda") -> torch.Tensor:
    """Config-2-style activations generated on the device: Gaussian with lognormal(0, 1) per-channel scale, bf16."""
    g = torch.Generator(device=device).manual_seed(seed)
    std = torch.exp(torch.randn(d, generator=g, device=device))
    out = torch.empty(tokens, d, dtype=torch.bfloat16, device=device)
    step = max(1, (1 << 28) // (4 * d))
    for a in range(0, tokens, step):
        b = min(tokens, a + step)
        out[a:b] = (torch.randn(b - a, d, generator=g, device=device) * std).to(torch.bfloat16)
    return out


def token_weights(tokens: int, seed: int, p: float = 0.08, big: float = 10.0, device="cuda") -> torch.Tensor:
    """Config 2's token weights: `big` on a Bernoulli(p) mask of tokens, 1 elsewhere (fp32)."""
    g = torch.Generator(device=device).manual_seed(seed)
    return torch.where(torch.rand(tokens, generator=g, device=device) < p, big, 1.0).float()


ACT_CHUNK = 16384  # activations are generated in fixed chunks of tokens, so any token shard matches the whole


def token_shard(tokens: int, rank: int, world: int, chunk: int = ACT_CHUNK) -> tuple[int, int]:
    """Tokens [lo, hi) of `rank`: whole generation chunks, split as evenly as possible."""
    chunks = (tokens + chunk - 1) // chunk
    return chunk * (chunks * rank // world), min(tokens, chunk * (chunks * (rank + 1) // world))


def stage_activations(tokens: int, d: int, seed: int, device="cuda", lo: int = 0, hi: int | None = None,
                      ref_noise: float = 0.02):
    """(x, x_ref) for tokens [lo, hi) of a stage: x Gaussian with lognormal(0, 1) channel scales (bf16), x_ref = x plus
    seeded noise of `ref_noise` × the channel scale (the reference stream differs by the upstream quantization error).
    Chunk c of the stage is drawn from seed (seed, c), so shards of any width reproduce the same tokens."""
    hi = tokens if hi is None else hi
    g = torch.Generator(device=device).manual_seed(seed)
    std = torch.exp(torch.randn(d, generator=g, device=device))
    x = torch.empty(hi - lo, d, dtype=torch.bfloat16, device=device)
    xr = torch.empty_like(x)
    for c in range(lo // ACT_CHUNK, (hi + ACT_CHUNK - 1) // ACT_CHUNK):
        a, b = c * ACT_CHUNK, min(tokens, (c + 1) * ACT_CHUNK)
        gc = torch.Generator(device=device).manual_seed(seed * 100003 + c)
        v = torch.randn(b - a, d, generator=gc, device=device) * std
        e = torch.randn(b - a, d, generator=gc, device=device) * (ref_noise * std)
        s, t = max(a, lo), min(b, hi)
        if s < t:
            x[s - lo:t - lo] = v[s - a:t - a].to(torch.bfloat16)
            xr[s - lo:t - lo] = (v[s - a:t - a] + e[s - a:t - a]).to(torch.bfloat16)
    return x, xr


def config3(tokens: int = 384 * 2048, device="cuda", lo: int = 0, hi: int | None = None, stages=None,
            weight_rows=None):
    """Config 3: one Qwen3-4B-class layer (q 4096, k/v 1024, o 2560 × 4096, gate/up 9728, down 2560 × 9728 rows ×
    inputs), bf16 weights N(0, 0.02²); config-2-style activations per stage (tokens [lo, hi) of `tokens`), token
    weights 10 on a Bernoulli(0.08) mask; per-row widths {1,2,3,4} w.p. {.15,.45,.30,.10} per 64-row group.
    Returns (stages, weights, acts, w, bits). `weight_rows` restricts weights to a row range per matrix (row shards)."""
    from .layer import qwen3_4b_stages, row_plan
    stages = stages or qwen3_4b_stages()
    weights, bits, acts = {}, {}, {}
    for si, s in enumerate(stages):
        for mi, (nm, rows) in enumerate(s.matrices):
            g = torch.Generator(device=device).manual_seed(1000 + 10 * si + mi)
            weights[nm] = (0.02 * torch.randn(rows, s.d, generator=g, device=device)).to(torch.bfloat16)
            bits[nm] = row_plan(rows, seed=2000 + 10 * si + mi)
        acts[s.name] = stage_activations(tokens, s.d, seed=3000 + si, device=device, lo=lo, hi=hi)
    hi = tokens if hi is None else hi
    w_all = token_weights(tokens, seed=7, device=device)
    return stages, weights, acts, w_all[lo:hi].contiguous(), bits
