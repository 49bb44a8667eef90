"""Row importance and GuidedQuant token weights on B200: the producers of the row plan and of the statistics' token
weights (ShinMegamiBoson/lookatmyquant, row_importance.py:57-93 and quantize.py:853-894).

Row importance: over calibration windows, each linear layer's output channel i gets E[g_i²]·E[y_i²], g the gradient at
that output of the log likelihood of tokens sampled from the model's own predictions (at the positions a weight selects;
the reference's are the positions that predict a digit), y the output. GuidedQuant: a calibration token's weight in a
matrix's statistics is the squared output gradient summed over the matrix's rows, normalised to mean 1 and clamped.

The model's forward and backward are the model's own (PyTorch autograd on its layers); the reductions the reference
writes as `pow(2).sum(...)` on fp64 copies of every output and gradient run in liblamq_b200.so (lamq_square_sums:
fp64 sums of squares over the tokens per channel, or over the channels per token, read straight from the bf16/fp32
tensors, deterministic). Sampling uses a device generator seeded as the reference's; `sampled` replaces it with given
tokens (to replay another run).
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from . import _lib
from ._lib import check, ptr, stream_ptr


def _rows(x: torch.Tensor) -> torch.Tensor:
    x = x.reshape(-1, x.shape[-1])
    if x.dtype not in (torch.float32, torch.bfloat16):
        x = x.float()
    return x if x.stride(-1) == 1 else x.contiguous()


def square_sums(x: torch.Tensor, col_acc: torch.Tensor | None = None, rows: bool = False):
    """fp64 sums of squares of x (..., C): adds Σ over the leading dimensions into col_acc (C fp64) and, with `rows`,
    returns each leading row's Σ over C (fp64)."""
    x = _rows(x)
    lib = _lib.load()
    n, c = x.shape
    row_out = torch.empty(n, dtype=torch.float64, device=x.device) if rows else None
    ws = None
    if col_acc is not None:
        ws = torch.empty(max(lib.lamq_square_sums_workspace_size(n, c), 8), dtype=torch.uint8, device=x.device)
    with torch.cuda.device(x.device):
        check(lib.lamq_square_sums(ptr(x), _lib.LAMQ_BF16 if x.dtype == torch.bfloat16 else _lib.LAMQ_F32, n, c,
                                   x.stride(0), ptr(col_acc), ptr(row_out), ptr(ws), 0 if ws is None else ws.numel(),
                                   stream_ptr(x.device)), "lamq_square_sums")
    return row_out


def importance_summary(imp: dict, sizes: dict | None = None) -> dict:
    """The statistics row_importance.py reports from each matrix's importance vector (:77-99): AM/GM, the bits per
    weight per-row widths are worth (half log2 of AM/GM), the share in the top 10 % of rows, the medians, and the
    weight-averaged bits worth (`sizes`: weights per matrix)."""
    res = {"matrices": {}}
    for k, v in imp.items():
        v = v.double()
        am, gm = float(v.mean()), float(v.log().mean().exp())
        top = v.sort(descending=True).values
        res["matrices"][k] = {"rows": len(v), "AM/GM": am / gm, "bits per weight per-row widths are worth":
                              0.5 * math.log2(am / gm),
                              "share of importance in the top 10% of rows":
                              float(top[:max(1, len(top) // 10)].sum() / top.sum())}
    vals = list(res["matrices"].values())
    res["median AM/GM"] = sorted(v["AM/GM"] for v in vals)[len(vals) // 2]
    if sizes:
        res["weight-averaged bits worth"] = sum(v["bits per weight per-row widths are worth"] * sizes[k]
                                                for k, v in res["matrices"].items()) / sum(sizes.values())
    return res


def row_importance(model, windows: torch.Tensor, mods: dict, position_weight: torch.Tensor | None = None,
                   seed: int = 0, sampled: list | None = None):
    """Each module's per-output-channel importance E[g²]·E[y²] (row_importance.py:57-93): for every window, the
    model's logits, tokens sampled from its own predictions (a device generator seeded `seed`, or `sampled[i]`), the
    log likelihood of the sampled tokens at the positions `position_weight` selects (1 everywhere by default)
    backpropagated; y² and g² of every module's output summed per channel over the tokens (fp64). Returns
    ({name: importance (fp64)}, sampled tokens per window)."""
    dev = next(model.parameters()).device
    gg = {k: torch.zeros(m.out_features, dtype=torch.float64, device=dev) for k, m in mods.items()}
    yy = {k: torch.zeros(m.out_features, dtype=torch.float64, device=dev) for k, m in mods.items()}

    def keep(key):
        def grad(g):
            square_sums(g, gg[key])

        def hook(m_, a_, o_):
            square_sums(o_.detach(), yy[key])
            o_.register_hook(grad)
        return hook

    hooks = [m.register_forward_hook(keep(k)) for k, m in mods.items()]
    gen = torch.Generator(device=dev).manual_seed(seed)
    drawn = []
    try:
        for i in range(len(windows)):
            x = windows[i:i + 1].to(dev)
            pw = torch.ones(x.shape, device=dev) if position_weight is None else position_weight[i:i + 1].to(dev)
            emb = model.get_input_embeddings()(x).detach().requires_grad_(True)
            lg = model(inputs_embeds=emb, use_cache=False).logits.float()
            with torch.no_grad():
                y = (sampled[i].to(dev) if sampled is not None else
                     torch.multinomial(F.softmax(lg[0], -1), 1, generator=gen)[:, 0])
            drawn.append(y)
            lp = F.log_softmax(lg[0], -1).gather(1, y[:, None])[:, 0]
            (lp * pw[0]).sum().backward()
            del lg, lp, emb
    finally:
        for h in hooks:
            h.remove()
    return {k: (gg[k] * yy[k]).clamp_min(1e-30) for k in mods}, drawn


def guided_weights(model, chunks: list, mods: dict, base: list, floor: float, ceiling: float = 100.0, seed: int = 0,
                   sampled: list | None = None):
    """GuidedQuant with one group per matrix (quantize.py:853-894): a calibration token's weight in a matrix's
    statistics is the squared gradient, at the matrix's output and summed over its rows, of the `base`-weighted log
    likelihood of tokens sampled from the model's own predictions. Per module name, one (windows, positions) fp32
    tensor per chunk, mean 1 and within [floor, ceiling] times the mean. `sampled[c][w]` replaces the draw.
    Returns (weights, sampled tokens per chunk and window)."""
    dev = next(model.parameters()).device
    out, s = {}, {k: [] for k in mods}

    def keep(k):
        def f(m, a, o):
            o.retain_grad()
            out[k] = o
        return f
    hooks = [m.register_forward_hook(keep(k)) for k, m in mods.items()]
    grads = [p.requires_grad for p in model.parameters()]
    for p in model.parameters():
        p.requires_grad_(False)
    gen = torch.Generator(device=dev).manual_seed(seed)
    embed = model.get_input_embeddings()
    drawn = []
    try:
        with torch.enable_grad():
            for c, x in enumerate(chunks):
                rows = {k: [] for k in mods}
                drawn.append([])
                for w in range(len(x)):
                    xi = x[w:w + 1].to(dev)
                    lp = torch.log_softmax(model(inputs_embeds=embed(xi).detach().requires_grad_(True),
                                                 use_cache=False).logits.float(), -1)
                    y = (sampled[c][w].to(dev).reshape(-1, 1) if sampled is not None else
                         torch.multinomial(lp.detach()[0].exp(), 1, generator=gen))
                    drawn[-1].append(y)
                    (lp[0].gather(-1, y)[:, 0] * base[c][w].to(dev)).sum().backward()
                    for k, o in out.items():
                        rows[k].append(square_sums(o.grad, rows=True).float().reshape(o.grad.shape[:-1]))
                    out.clear()
                    del lp, y
                for k in mods:
                    s[k].append(torch.cat(rows[k]))
    finally:
        for h in hooks:
            h.remove()
        for p, g in zip(model.parameters(), grads):
            p.requires_grad_(g)
    res = {}
    for k, v in s.items():
        w = torch.cat(v).double()
        w = (w / w.mean()).clamp(floor, ceiling)
        res[k] = (w / w.mean()).float().split(len(chunks[0]))
    return res, drawn
