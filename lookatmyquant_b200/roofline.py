"""Every hot-path kernel timed alone at its configuration's size, against the roofline that bounds it.

`python -m lookatmyquant_b200.roofline [--only a14 ...] [--out FILE]` prints one JSON record per kernel (and a markdown table): the
row of the path it serves, the shape, the device time (CUDA events on the launching stream, median of several
launches after a warm-up, L2 flushed before each), the algorithmic work, the achieved rate and its fraction of the
peak. Peaks: HBM copy and bf16 GEMM from MEASURED_PEAKS.json (measured on this pool's B200s), fp32 lanes =
148 SMs × 128 lanes × 1.965 GHz, fp64 tensor = 36.6 TFLOP/s (a loop of mma.sync m16n8k16 f64 on this pool; cuBLAS
DGEMM reaches 35.8). Inputs are seeded synthetic data with the configurations' shapes.
"""

from __future__ import annotations

import argparse
import math
import json
import statistics
from pathlib import Path

import torch

PEAKS_FILE = Path(__file__).resolve().parents[1] / "MEASURED_PEAKS.json"
FP32_LANES_T = 148 * 128 * 1.965e9 / 1e12
FP64_TENSOR_TF = 36.6
FP64_ADD_T = 18.6  # scalar fp64 adds per second (one per FMA slot: ~37 TFLOP/s of FMAs)


def _peaks() -> dict:
    if PEAKS_FILE.exists():
        d = json.loads(PEAKS_FILE.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


class Timer:
    """Median device time of fn() on the current stream, after a warm-up, with L2 flushed (a 256 MB write)
    before each launch."""

    def __init__(self, device):
        self.flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)

    def __call__(self, fn, reps: int = 5) -> float:
        fn()
        torch.cuda.synchronize()
        out = []
        for _ in range(reps):
            self.flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            b.synchronize()
            out.append(a.elapsed_time(b))
        return statistics.median(out)


def _record(row, kernel, shape, ms, work, unit, peak, note="", bound=None):
    rate = work / (ms * 1e-3)
    scale = {"TFLOP/s": 1e12, "GB/s": 1e9, "T lane-ops/s": 1e12, "T fp64 add/s": 1e12}[unit]
    achieved = rate / scale
    return {"row": row, "kernel": kernel, "shape": shape, "ms": round(ms, 4), "achieved": round(achieved, 2),
            "unit": unit, "peak": peak, "frac": round(achieved / peak, 3), "bound": bound or unit, "note": note}


def spd(n: int, device, seed: int = 0) -> torch.Tensor:
    """A positive definite n × n fp64 matrix with lognormal channel scales (setup only, cuBLAS)."""
    g = torch.Generator(device=device).manual_seed(seed)
    A = torch.randn(2 * n, n, dtype=torch.float64, device=device, generator=g)
    A = A * torch.exp(torch.randn(n, dtype=torch.float64, device=device, generator=g))
    return A.T @ A / (2 * n)


def trellis_paths(rows: int, n: int, k: int, device, seed: int) -> torch.Tensor:
    """Random row trellis paths from state 0 (s_t = (s_{t-1}·2^k + b_t) mod 4096), int64, built without a loop
    over t: s_t is the last ⌈12/k⌉ symbols, shifted into place."""
    g = torch.Generator(device=device).manual_seed(seed)
    b = torch.randint(0, 1 << k, (rows, n), generator=g, device=device, dtype=torch.int64)
    s = torch.zeros_like(b)
    for i in range((12 + k - 1) // k):
        sh = torch.zeros_like(b)
        sh[:, i:] = b[:, :n - i] if i else b
        s |= sh << (k * i)
    return s & 4095


def packed_layer(device, seed: int = 0):
    """A config-3 layer packed as opgraph-packed-1 trellis row groups (the row plan's widths, random valid paths,
    the shipped k = 1..4 tables): {matrix: (TrellisProduct, input width, tensors, meta, stage)}."""
    from . import artifact
    from .codes import stacked_tables
    from .layer import qwen3_4b_stages, row_plan
    tables = stacked_tables(12, 256, device).to(torch.float32).reshape(-1).contiguous()
    out = {}
    for si, s in enumerate(qwen3_4b_stages()):
        for mi, (nm, rows) in enumerate(s.matrices):
            bits = row_plan(rows, seed=2000 + 10 * si + mi).to(device)
            states = torch.empty(rows, s.d, dtype=torch.int64, device=device)
            groups = []
            for k in (1, 2, 3, 4):
                idx = torch.nonzero(bits == k).flatten()
                if idx.numel() == 0:
                    continue
                states[idx] = trellis_paths(idx.numel(), s.d, k, device, seed + 97 * k + mi) + 4096 * (k - 1)
                groups.append({"rows": idx.cpu(), "bits": k, "table_index": k - 1})
            g = torch.Generator(device=device).manual_seed(seed + 5 + mi)
            scales = (0.02 * (1 + torch.rand(rows, generator=g, device=device))).float()
            # the matrices of a stage read one input through the same signs (one in_seed per stage)
            entry = {"states": states, "scales": scales, "in_seed": 1000 * si + 1, "table": tables,
                     "row_groups": groups}
            tensors, meta = artifact.encode_entry(nm, entry)
            out[nm] = (artifact.TrellisProduct(tensors, meta, device), s.d, tensors, meta, s.name)
    return out


def run(device="cuda", log=print, only=None) -> list:
    from . import _lib, artifact, codes
    from .artifact import decode_rotated, pack_trellis
    from .frame import Environment
    from .hessian import Statistics
    from .kl import KLReference
    from .linalg import CrossTarget, cholesky_inverse_lower, env_factor, ridge
    from .rotation import Rotation
    from .workloads import stage_activations, token_weights
    dev = torch.device(device)
    _lib.load()
    pk = _peaks()
    hbm, bf16 = pk["hbm_gbs"], pk["bf16_tflops"]
    timer = Timer(dev)
    recs = []

    def add(r):
        recs.append(r)
        log(json.dumps(r))

    def want(row):
        return only is None or row in only

    # a1: H and D statistics (tcgen05), 65,536 config-2 tokens, token weights 10 on 8 %
    for d in ((2560, 9728) if want("a1") else ()):
        x, xr = stage_activations(65536, d, seed=3000, device=dev)
        w = token_weights(65536, seed=7, device=dev)
        nw = int((w != 1).sum())

        def stats():
            st = Statistics(d, cross=True, device=dev)
            st.add(x, w, xr)
        ms = timer(stats)
        flops = 2.0 * (65536 + nw) * (d * (d + 1) / 2 + d * d)
        add(_record("a1", "xtx_pair_kernel (H triangle + D, weighted tokens in their own pass)",
                    f"65536 tokens x {d}", ms, flops, "TFLOP/s", bf16, "executed flops", "tensor"))
        del x, xr

    g = torch.Generator(device=dev).manual_seed(1)
    # a5, a2: the two fp64 factorizations and the QEP map of the d = 9728 stage (down_proj, 2560 rows)
    n, rows = 9728, 2560
    H = spd(n, dev) if want("a2") or want("a5") or want("a3") else None
    if want("a5"):
        ms = timer(lambda: env_factor(H)[0], reps=3)
        add(_record("a5", "lamq_env_factor (flip, recursive Cholesky + inverse on DMMA)", f"n = {n}", ms,
                    2.0 * n ** 3 / 3, "TFLOP/s", FP64_TENSOR_TF, "n³/3 multiply-adds", "fp64 tensor"))
    if want("a2"):
        ms = timer(lambda: cholesky_inverse_lower(ridge(H, 0.1), deferred=True)[0], reps=3)
        add(_record("a2", "lamq_cholesky_inverse_lower (the QEP factor)", f"n = {n}", ms, 2.0 * n ** 3 / 3,
                    "TFLOP/s", FP64_TENSOR_TF, "n³/3 multiply-adds", "fp64 tensor"))
        D = 0.05 * spd(n, dev, seed=2)
        W = 0.02 * torch.randn(rows, n, dtype=torch.float64, device=dev, generator=g)
        qep = CrossTarget(H, D, 0.5, 0.1, rows=rows)
        ms = timer(lambda: qep.apply(W), reps=3)
        add(_record("a2", "lamq_cross_apply (W·D, then two triangular products)", f"{rows} x {n}", ms,
                    4.0 * rows * n * n, "TFLOP/s", FP64_TENSOR_TF, "2·rows·n² + 2·rows·n²/2 ·2 flops",
                    "fp64 tensor"))
        del D, qep

    if want("dgemm"):  # the recursion's top-level product size at n = 9728 (the 128 x 128 CTA tile)
        from .linalg import gemm
        m = n // 2
        A = torch.randn(m, m, dtype=torch.float64, device=dev, generator=g)
        B = torch.randn(m, m, dtype=torch.float64, device=dev, generator=g)
        ms = timer(lambda: gemm(A, B), reps=3)
        add(_record("a5", "dgemm_kernel (128 x 128 tiles, mma.sync f64)", f"{m}^3", ms, 2.0 * m ** 3, "TFLOP/s",
                    FP64_TENSOR_TF, "the factorizations' largest products", "fp64 tensor"))
        del A, B

    if want("a3"):  # the randomized Hadamard transform of a stage's targets (9728 x 2560) and of H (9728²)
        def adds_per_row(n_):
            """Additions per row: a Sylvester factor (a power-of-two order, applied by butterflies) costs log2 of its
            order per element, a Paley one its order (dense signed sums)."""
            A, B = codes.hadamard_factors(n_)
            na, nb = int(A.shape[0]), int(B.shape[0])
            sylvester = lambda m: m & (m - 1) == 0 and m > 1
            ca = math.log2(na) if sylvester(na) else na
            cb = math.log2(nb) if sylvester(nb) and torch.equal(B, codes._sylvester(int(math.log2(nb)))) else nb
            return na, nb, float(na * nb) * (ca + cb)
        for n_, rows_ in ((2560, 9728), (9728, 2560)):
            rot = Rotation(n_, 301, dev)
            X = 0.02 * torch.randn(rows_, n_, dtype=torch.float64, device=dev, generator=g)
            ms = timer(lambda: rot.rows(X))
            na, nb, per_row = adds_per_row(n_)
            add(_record("a3", "rht_rows_kernel (A·V·Bᵀ: butterflies for the Sylvester factor, signed sums for Paley)",
                        f"{rows_} x {n_} ({na} x {nb})", ms, rows_ * per_row, "T fp64 add/s", FP64_ADD_T,
                        f"{16.0 * X.numel() / (ms * 1e-3) / 1e9:.0f} GB/s of HBM", "fp64 pipe"))
            del X
        rot9 = Rotation(n, 301, dev)
        ms = timer(lambda: rot9.conj(H))
        na, nb, per_row = adds_per_row(n)
        add(_record("a3", "rht_rows_kernel x2 + transpose (R·H·Rᵀ)", f"{n}²", ms, 2.0 * n * per_row,
                    "T fp64 add/s", FP64_ADD_T, "two row passes", "fp64 pipe"))

    if want("a6"):  # the fused row-trellis sweep (4096 x 2560 at k = 2, and the down_proj shape)
        for r_, n_, k in ((4096, 2560, 2), (2560, 9728, 2)):
            env = Environment(spd(n_, dev, seed=3))
            Xs = 0.02 * torch.randn(r_, n_, dtype=torch.float64, device=dev, generator=g)
            S = Xs.pow(2).mean(1).sqrt()
            code = codes.RowTrellisCode(12, k)
            ms = timer(lambda: codes._row_trellis_sweep(Xs, S, env, code), reps=3)
            wins = sum(min(16, n_ - j) + min(8, max(0, n_ - j - 16)) for j in range(0, n_, 16))
            add(_record("a6+a7", "sweep_run_kernel + per-run DGEMM (fused row-trellis LDLQ sweep)",
                        f"{r_} x {n_}, k = {k}", ms, 3.0 * wins * 4096 * r_, "T lane-ops/s", FP32_LANES_T,
                        "3 fp32 ops per state per trellis step (compares not counted)", "fp32 issue"))
            del env, Xs

    if want("a7"):  # the Viterbi alone: 65,536 windows of 24 at k = 2
        vals = codes.trellis_values(12, 2, 256)
        xs = torch.randn(65536, 24, dtype=torch.float32, device=dev, generator=g)
        ms = timer(lambda: codes.viterbi(xs, vals, 12, 2))
        add(_record("a7", "viterbi_kernel (one warp per sequence)", "65536 x 24, k = 2", ms,
                    3.0 * 24 * 4096 * 65536, "T lane-ops/s", FP32_LANES_T, "3 fp32 ops per state per step",
                    "fp32 issue"))

    if want("a8"):  # the column-trellis sweep of the measure path (SmolLM2 gate_proj 2560 x 960, T = 320)
        env = Environment(spd(960, dev, seed=4))
        Xc = 0.02 * torch.randn(2560, 960, dtype=torch.float64, device=dev, generator=g)
        S = Xc.pow(2).mean(1).sqrt()
        tcode = codes.TrellisCode(12, 2, T=320)
        ms = timer(lambda: codes._col_trellis_sweep(Xc, S, env, tcode), reps=3)
        add(_record("a8", "lamq_ldlq_coltrellis (column Viterbi per block + refit)", "2560 x 960, T = 320, k = 2",
                    ms, 3.0 * 2560 * 960 * 4096, "T lane-ops/s", FP32_LANES_T, "3 fp32 ops per state per step",
                    "fp32 issue"))

    if want("a13"):  # the KL head of one probe (16,384 positions, V = 49,152, d = 960)
        P_, V_, d_ = 16384, 49152, 960
        E = (0.02 * torch.randn(V_, d_, device=dev, generator=g)).to(torch.bfloat16)
        h_ref = torch.randn(P_, d_, device=dev, generator=g).to(torch.bfloat16)
        h = (h_ref.float() + 0.05 * torch.randn(P_, d_, device=dev, generator=g)).to(torch.bfloat16)
        ref = KLReference(h_ref, E)
        ms = timer(lambda: ref.kl(h))
        add(_record("a13", "kl_head_kernel (LM head GEMM + log-softmax + KL, no logits written)",
                    f"{P_} x {V_} x {d_}", ms, 2.0 * P_ * V_ * d_, "TFLOP/s", bf16,
                    f"also streams the stored distribution: {4 * P_ * V_ / (ms * 1e-3) / 1e9:.0f} GB/s", "tensor"))
        del ref, E

    if want("a14"):  # a config-3 layer packed at the row plan's widths
        layer = packed_layer(dev)
        weights = sum(v[0].m * v[0].n for v in layer.values())
        code_bytes = sum(t.numel() * t.element_size() for v in layer.values() for key, t in v[2].items()
                         if not key.endswith(".signs"))
        first = {}  # the first matrix of each stage rotates the stage's input for all of them
        stages = {}  # the matrices of each stage: one grouped product launch reads the stage's rotated input
        for nm, v in layer.items():
            first.setdefault(v[4], nm)
            stages.setdefault(v[4], []).append(v[0])
        for batch in (1, 16, 2048):
            xs = {st: torch.randn(batch, layer[nm][1], device=dev, generator=g).to(torch.bfloat16)
                  for st, nm in first.items()}

            def product():
                xr = {st: layer[nm][0].rotate(xs[st]) for st, nm in first.items()}
                return artifact.product_layer([(ps, xr[st]) for st, ps in stages.items()])
            if batch >= artifact.GEMM_PRODUCT_VECTORS:
                ms = timer(product)
                add(_record("a14", "input rotation per stage + trellis_gemm_kernel (decode fused into tcgen05 GEMM)",
                            f"layer, batch {batch}", ms, 2.0 * batch * weights, "TFLOP/s", bf16,
                            "weights decoded from the packed states into shared memory, never written", "tensor"))
                xr = {st: layer[nm][0].rotate(xs[st]) for st, nm in first.items()}
                ms = timer(lambda: artifact.product_layer([(ps, xr[st]) for st, ps in stages.items()]))
                add(_record("a14", "trellis_gemm_kernel alone (rotated inputs given, the layer's groups in 2 launches)",
                            f"layer, batch {batch}", ms, 2.0 * batch * weights, "TFLOP/s", bf16,
                            f"codes {code_bytes / 1e6:.1f} MB per pass", "tensor"))
                continue
            # launch-bound at small batches: the whole layer's product is replayed as one CUDA graph
            side = torch.cuda.Stream(device=dev)
            side.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(side):
                product()
                product()
            torch.cuda.current_stream(dev).wait_stream(side)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, capture_error_mode="relaxed"):
                product()
            ms = timer(graph.replay)
            io = sum(2 * x.numel() for x in xs.values()) + sum(4 * batch * v[0].m for v in layer.values())
            add(_record("a14", "trellis_product_groups_kernel per stage + one input rotation per stage (one CUDA graph)",
                        f"layer ({weights / 1e6:.1f} M weights), batch {batch}", ms, code_bytes + io, "GB/s", hbm,
                        f"{weights * batch / (ms * 1e-3) / 1e12:.2f} T weight-products/s", "hbm"))
            xr = {st: layer[nm][0].rotate(xs[st]) for st, nm in first.items()}
            ms = timer(lambda: [artifact.product_rotated(ps, xr[st]) for st, ps in stages.items()])
            add(_record("a14", "trellis_product_groups_kernel alone (rotated inputs given, one launch per stage)",
                        f"layer, batch {batch}", ms, code_bytes + io, "GB/s", hbm,
                        f"{weights * batch / (ms * 1e-3) / 1e12:.2f} T weight-products/s", "hbm"))
            del graph
        ms = timer(lambda: [decode_rotated(v[2], v[3]) for v in layer.values()])
        add(_record("a14", "unpack_trellis_kernel (decode_rotated: table·scale, fp32)", "layer", ms,
                    code_bytes + 4.0 * weights, "GB/s", hbm, "codes read, fp32 weights written", "hbm"))

    if want("a15"):
        st = trellis_paths(9728, 2560, 2, dev, 11).to(torch.int16)
        ms = timer(lambda: pack_trellis(st, 2))
        add(_record("a15", "pack_trellis_kernel (path check + k-bit reversed stream)", "9728 x 2560, k = 2", ms,
                    2.0 * st.numel() + st.numel() * 2 / 8, "GB/s", hbm, "int16 states read, codes written", "hbm"))
    return recs


def table(recs) -> str:
    lines = ["| row | kernel | shape | ms | achieved | peak | frac | note |", "|---|---|---|---|---|---|---|---|"]
    for r in recs:
        lines.append(f"| {r['row']} | {r['kernel']} | {r['shape']} | {r['ms']} | {r['achieved']} {r['unit']} | "
                     f"{r['peak']} | {r['frac']} | {r['note']} |")
    return "\n".join(lines)


def main():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--out", default=None, help="write the records as JSON")
    ap.add_argument("--only", nargs="+", default=None, help="rows to measure (a1 a2 a3 a5 dgemm a6 a7 a8 a13 a14 a15)")
    a = ap.parse_args()
    recs = run(only=set(a.only) if a.only else None)
    print(table(recs), flush=True)
    if a.out:
        Path(a.out).write_text(json.dumps(recs, indent=1))


if __name__ == "__main__":
    main()
