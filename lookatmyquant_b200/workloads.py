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
