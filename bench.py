"""Benchmark of the quantization-build hot path on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload config1] [--impl ours|reference]

Workloads (seeded synthetic inputs, resident in HBM before timing):
  config1  one SmolLM2-360M gate_proj (2560 × 960) built to a 2-bit row trellis with block LDLQ: rotation, row scales,
           environment (U), the fused Viterbi sweep, dequantization. Metric: seconds per build.

`value` is device time per step (CUDA events, L2 flushed before every step, max over ranks); `e2e` is the same step
through the public API with the inputs copied from pinned host memory and the result read back inside the timed
region. `--impl reference` times the CPU oracle port of the reference's algorithm on the host cores.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402
import torch  # noqa: E402

PEAKS = ROOT / "MEASURED_PEAKS.json"
FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "sm_max_mhz": 1965.0}
SMS = 148
FP32_LANES = 128


# DRAM bytes (read + write) of the statistics kernels per calibration token, summed over the 16 launches of one
# config-3 layer (H and D of every stage, and of its weighted tokens) and the fixed-order reductions of their last
# windows: ncu dram__bytes_read.sum + dram__bytes_write.sum of every xtx and last_window launch of
# `python -m lookatmyquant_b200.layer --tokens 65536` (31.58 GB / 65,536 tokens). The kernel's traffic per token does
# not depend on the token count (each launch streams its tokens once through the same tile order), so a launch at any
# token count moves this many bytes per token.
XTX_DRAM_BYTES_PER_TOKEN = 481_864
XTX_LAUNCHES_PER_LAYER = 16


def peaks():
    if PEAKS.exists():
        d = json.loads(PEAKS.read_text())
        d["source"] = "measured"
        return d
    return dict(FALLBACK, source="fallback")


class Clocks:
    """Samples nvidia-smi clocks and throttle reasons while the timed region runs."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index, self.proc, self.lines = index, None, []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ----------------------------------------------------------------------------- workloads


class Config1:
    name = "config1"
    metric = "s per single-linear LDLQ + 2-bit row-trellis build (SmolLM2-360M gate_proj 2560x960)"
    unit = "s"

    def __init__(self, device):
        from lookatmyquant_b200 import codes
        from lookatmyquant_b200.workloads import config1
        self.codes = codes
        W, H, self.seed, self.in_seed = config1()
        self.W_host = W.pin_memory()
        self.H_host = H.pin_memory()
        self.W, self.H = W.to(device), H.to(device)
        self.code = codes.RowTrellisCode(12, 2, T=256, width=16, look=8)
        self.device = device
        self.m, self.n = W.shape

    def step(self, W=None, H=None):
        return self.codes.ldlq_words([self.W if W is None else W], self.H if H is None else H, self.code,
                                     [self.seed], in_seed=self.in_seed, out_rot=False, device=self.device)[0]

    def e2e_step(self):
        W = self.W_host.to(self.device, non_blocking=True)
        H = self.H_host.to(self.device, non_blocking=True)
        word = self.step(W, H)
        states = word.states.to("cpu", non_blocking=False)
        scales = word.scales.to("cpu")
        return states, scales

    def e2e_bytes(self):
        return self.W_host.numel() * 8 + self.H_host.numel() * 8, self.m * self.n * 2 + self.m * 8

    def sweep_algorithmic(self):
        """Per sweep launch: bytes the kernel must move (targets read and written back, states and settled values
        written, U's upper triangle read once) and trellis edges it must evaluate (every window of 16 + 8 columns:
        (win − 1) add-compare-select steps over 4096 predecessor edges, plus the final 4096 costs)."""
        m, n = self.m, self.n
        bytes_ = m * n * (8 + 8 + 2 + 8) + 8 * n * (n + 1) // 2 + m * 8
        edges = 0
        for j in range(0, n, 16):
            w = min(16, n - j)
            win = w + min(8, n - j - w)
            edges += win * 4096
        return bytes_, edges * m

    def prepare_e2e(self):
        pass

    def config(self):
        return {"workload": self.name, "rows": self.m, "cols": self.n, "bits": 2,
                "trellis": "L=12 k=2 (reference table)", "width": 16, "look": 8, "lazy": 128}

    def roofline(self, pk):
        kms = sweep_kernel_ms(self)
        algo_bytes, edges = self.sweep_algorithmic()
        return sweep_roofline(kms, algo_bytes, edges, pk)

    def cpu_sample(self, threads):
        return config1_cpu_sample(threads, self.W_host.numpy(), self.H_host.numpy(), self.in_seed,
                                  self.code.values.numpy())


class Config3:
    """One Qwen3-4B-class decoder layer built to a 1-4-bit row plan, tokens sharded across ranks
    for H/D (one all-reduce per stage), rows sharded for the sweep, states gathered at the end."""
    name = "config3"
    metric = "s per Qwen-4B-class layer build"
    unit = "s"

    def __init__(self, device, tokens=384 * 2048, group=None):
        from lookatmyquant_b200.workloads import config3
        self.device, self.group = device, group
        self.world = group.size() if group is not None else 1
        self.rank = group.rank() if group is not None else 0
        self.tokens = tokens
        from lookatmyquant_b200.workloads import token_shard
        lo, hi = token_shard(tokens, self.rank, self.world)
        self.lo, self.hi = lo, hi
        self.stages, self.weights, self.acts, self.w, self.bits = config3(tokens, device=device, lo=lo, hi=hi)
        self.m = sum(r for s in self.stages for _, r in s.matrices)
        self.n_weights = sum(r * s.d for s in self.stages for _, r in s.matrices)
        self.stage_ms = {}

    def step(self, timed=False):
        from lookatmyquant_b200.hessian import Statistics
        from lookatmyquant_b200.layer import build_stage, build_stages_sharded, stacked_tables
        tables = stacked_tables(12, 256, self.device)
        out = {}
        if self.world >= 2:  # every stage's statistics first, the stages' factorizations on rank pairs, beside the sweeps
            stats = []
            for s in self.stages:
                x, xr = self.acts[s.name]
                st = Statistics(s.d, cross=True, device=self.device)
                st.add(x, self.w, xr)
                stats.append(st)
            out = build_stages_sharded(self.stages, self.weights, stats, self.bits, 0, self.group, True, tables,
                                       self.tokens)
            self.gather(out)
            return out
        for s in self.stages:
            if timed:
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
            x, xr = self.acts[s.name]
            out[s.name] = build_stage(s, self.weights, x, xr, self.w, self.bits, 0, self.group, True, tables,
                                      self.tokens)
            if timed:
                b.record()
                self.stage_ms.setdefault(s.name, []).append((a, b))
        if self.group is not None:
            self.gather(out)
        return out

    def gather(self, out):
        """All ranks end with every matrix's states (int16): one all-gather per stage of padded row shards."""
        for s in self.stages:
            parts = [out[s.name].states[nm] for nm, _ in s.matrices if nm in out[s.name].states]
            mine = torch.cat(parts) if parts else torch.empty(0, s.d, dtype=torch.int16, device=self.device)
            total = sum(r for _, r in s.matrices)
            cap = ((total + 63) // 64 + self.world - 1) // self.world * 64
            buf = torch.zeros(cap, s.d, dtype=torch.int16, device=self.device)
            buf[:len(mine)] = mine
            allb = torch.empty(self.world * cap, s.d, dtype=torch.int16, device=self.device)
            # collectives have no int16 type: the shards travel as bytes
            torch.distributed.all_gather_into_tensor(allb.view(torch.uint8), buf.view(torch.uint8), group=self.group)

    def e2e_step(self):
        """The build from host memory through the public API (layer.build_layer_from_host): every stage's weights and
        activations copied from pinned host buffers inside the timed region (overlapped with the compute), the states
        and scales read back."""
        from lookatmyquant_b200.layer import build_layer_from_host
        out = build_layer_from_host(self.stages, self.host_weights, self.host_acts, self.host_w, self.bits, 0,
                                    self.group, self.tokens, device=self.device)
        return [t for r in out.values() for nm in r.states for t in (r.states[nm], r.scales[nm])]

    def prepare_e2e(self):
        self.host_acts = {k: (a.cpu().pin_memory(), b.cpu().pin_memory()) for k, (a, b) in self.acts.items()}
        self.host_weights = {k: v.cpu().pin_memory() for k, v in self.weights.items()}
        self.host_w = self.w.cpu().pin_memory()

    def e2e_bytes(self):
        h2d = sum(a.numel() * 2 + b.numel() * 2 for a, b in self.acts.values())
        h2d += sum(v.numel() * 2 for v in self.weights.values()) + self.w.numel() * 4
        rows_mine = self.m // self.world
        d2h = sum(r * s.d * 2 + r * 8 for s in self.stages for _, r in s.matrices) // self.world
        return h2d, d2h

    def config(self):
        return {"workload": self.name, "model": "Qwen3-4B-class layer (hidden 2560, 32/8 heads of 128, MLP 9728)",
                "matrices": {nm: [r, s.d] for s in self.stages for nm, r in s.matrices}, "weights": self.n_weights,
                "calibration_tokens": self.tokens, "token_weights": "10 on Bernoulli(0.08), else 1",
                "row_plan": "per 64-row group widths {1,2,3,4} w.p. {.15,.45,.30,.10}",
                "trellis": "L=12 reference e-means tables (4096 states) for every width",
                "qep_alpha": 0.5, "width": 16, "look": 8, "lazy": 128,
                "parallelism": f"tokens x{self.world} (H/D all-reduce), rows x{self.world}, " +
                               ("each stage's two factorizations on ranks 0/1, broadcast" if self.world < 2 else
                                "the stages' factorizations on rank pairs beside the other stages' sweeps, broadcast"),
                "l2": "inputs (60 GB of activations) far larger than L2"}

    def roofline(self, pk):
        """Both kernel families, timed alone on the stream they run on: the Hessian/QEP tensor-core contraction and
        the fused Viterbi sweep; the one with the larger share of the layer is reported as the roofline."""
        from lookatmyquant_b200.hessian import Statistics
        from lookatmyquant_b200.layer import Environment, Rotation, cross_target, stacked_tables, sweep_rows
        tables = stacked_tables(12, 256, self.device)
        h_ms = sw_ms = 0.0
        h_flop = 0.0
        self.h_accum = {}
        edges = 0
        sweep_bytes = 0
        for s in self.stages:
            x, xr = self.acts[s.name]
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            st = Statistics(s.d, cross=True, device=self.device)
            a.record()
            st.add(x, self.w, xr)
            b.record()
            b.synchronize()
            h_ms += a.elapsed_time(b)
            ntok = x.shape[0]
            # algorithmic flops: H's triangle d(d+1)/2 and D's d^2 entries, 2 flops per token each (the weighted
            # tokens' second pass, 8 % more work the kernel executes, is not counted)
            h_flop += 2.0 * ntok * (s.d * (s.d + 1) / 2 + s.d * s.d)
            # BASELINE config 2's count: 2·N·d² for H (and as much again for D), N this rank's tokens
            self.h_accum[s.name] = {"d": s.d, "tokens": ntok, "ms": a.elapsed_time(b),
                                    "tflops_2Nd2": 2.0 * 2.0 * ntok * s.d * s.d / (a.elapsed_time(b) * 1e-3) / 1e12}
            H, D = st.finalize(self.tokens)
            rot = Rotation(s.d, 301, self.device)
            env = Environment(rot.conj(H))
            rows = sum(r for _, r in s.matrices) // self.world
            X = torch.randn(rows, s.d, dtype=torch.float64, device=self.device) * 0.02
            S = X.pow(2).mean(1).sqrt()
            kb = torch.cat([self.bits[nm] for nm, _ in s.matrices])[:rows].to(self.device)
            a.record()
            sweep_rows(X, S, env, kb, tables)
            b.record()
            b.synchronize()
            sw_ms += a.elapsed_time(b)
            wins = sum(min(16, s.d - j) + min(8, max(0, s.d - j - 16)) for j in range(0, s.d, 16))
            edges += wins * 4096 * rows
            sweep_bytes += rows * s.d * (8 + 8 + 2 + 8) + 8 * s.d * (s.d + 1) // 2
        h_tflops = h_flop / (h_ms * 1e-3) / 1e12
        ntok = self.acts[self.stages[0].name][0].shape[0]
        traffic = XTX_DRAM_BYTES_PER_TOKEN * ntok / XTX_LAUNCHES_PER_LAYER  # per launch, like `achieved`
        hess = {"kernel": "xtx_pair_kernel (tcgen05 H/D accumulation)", "bound": "tensor", "achieved": h_tflops,
                "peak": pk["bf16_tflops"], "unit": "TFLOP/s", "frac": h_tflops / pk["bf16_tflops"],
                "traffic": traffic, "traffic_unit": "bytes per launch (ncu, scaled by tokens)",
                "kernel_ms": h_ms, "peak_source": pk["source"],
                "note": "algorithmic flops: H's upper triangle and D in full over every token once (the weighted tokens' "
                        "extra pass not counted); traffic: ncu DRAM bytes of the shipped kernel at 65,536 tokens "
                        "(profiles/xtx_pair_kernel_dram_layer65k.md) scaled by tokens"}
        sw = sweep_roofline(sw_ms, sweep_bytes, edges, pk)
        main, other = (hess, sw) if h_ms >= sw_ms else (sw, hess)
        main = dict(main)
        main["other"] = other
        return main

    def cpu_sample(self, threads):
        return config3_cpu_sample(threads, self.tokens)


_ROTATIONS = {}
GROUPS_PER_MATRIX = 4  # ldlq_words calls per matrix under a 1-4-bit row plan: one per width (quantize.py:530-565)


def _dense_rotation(n, seed=301):
    """The reference's dense rht(n) (codes.py:129-132) from the oracle, formed once per width outside timed work."""
    from oracle import core as O
    if (n, seed) not in _ROTATIONS:
        _ROTATIONS[(n, seed)] = O.rht(n, seed)
    return _ROTATIONS[(n, seed)]


def _words_seconds(W, R, U, dead, values):
    """Seconds of the reference's per-row word work (ldlq_words, codes.py:425-462) on the oracle for the rows of W:
    X = W·R_inᵀ, the row scales, the sweep (a Viterbi per block, the refit) and W_q = (S⊙V)·R_in. The sample's matrix
    products are small, so BLAS keeps one thread and the OpenMP Viterbi the cores (two thread pools spinning against
    each other made small samples several times slower than their rows' share of a full call)."""
    from threadpoolctl import threadpool_limits
    from oracle import core as O
    with threadpool_limits(limits=1, user_api="blas"):
        t0 = time.perf_counter()
        X = W @ R.T
        S = O.row_scale(X)
        _, settled, _ = O.row_trellis_sweep(X, S, U, dead, values, 12, 2)
        (settled * S[:, None]) @ R
        return time.perf_counter() - t0


def words_fit(W, R, U, dead, values, r1=16, r2=128):
    """(seconds per call, seconds per row) of the word work at W's width: a line through its times on the first r1
    and r2 rows of W (a call's cost is one part per block of columns, whatever its rows, plus one part per row).
    Times out of order (noise) give the larger sample's time per row and nothing per call."""
    t1 = _words_seconds(W[:r1], R, U, dead, values)
    t2 = _words_seconds(W[:r2], R, U, dead, values)
    if t2 <= t1:
        return 0.0, t2 / r2
    per_row = (t2 - t1) / (r2 - r1)
    return max(t1 - per_row * r1, 0.0), per_row


def _warm_oracle(values):
    """Loads the oracle's C Viterbi (and builds it if needed) before anything is timed."""
    from oracle import core as O
    O.viterbi(np.zeros((1, 2)), values, 12, 2)


def config1_cpu_sample(threads, W, H, in_seed, values):
    """The reference's path for one word (config 1) on the oracle: R·H·Rᵀ and the environment once (all threads),
    then the word work of one call over all of W's rows, from its line fitted on 64 and 512 rows."""
    from oracle import core as O
    O.set_threads(threads)
    _warm_oracle(values)
    R = _dense_rotation(W.shape[1], in_seed)
    t0 = time.perf_counter()
    U, dead, _ = O.environment(R @ H @ R.T)
    t_fix = time.perf_counter() - t0
    per_call, per_row = words_fit(W, R, U, dead, values, 64, 512)
    t_w = per_call + per_row * W.shape[0]
    return t_fix + t_w, (f"oracle on {threads} host threads: R·H·Rᵀ + environment ({t_fix:.2f} s), then the word's "
                         f"sweep fitted on 64 and 512 of {W.shape[0]} rows: {per_call:.2f} s per call + "
                         f"{per_row * 1e3:.1f} ms per row ({t_w:.0f} s)")


_FIXED_CACHE = {}


def _ldlq_call_fixed_seconds(n):
    """Seconds of the work the reference's ldlq_words repeats on every call at input width n, whatever the call's
    rows (codes.py:425-439 with GPU_SWEEP off, torch on the CPU as the reference runs it): the dense rht(n), the
    rotated statistics R·H·Rᵀ and the Environment's three factorizations (frame.py:515-522)."""
    rng = np.random.default_rng(n)
    A = torch.from_numpy(rng.standard_normal((n + 64, n)))
    H = A.T @ A / (n + 64)
    t0 = time.perf_counter()
    R = torch.from_numpy(_dense_rotation(n, 301))  # formed by the reference per call (torch.kron), here from cache
    Hr = R @ H @ R.T
    Hr += 0.01 * torch.mean(torch.diag(Hr)) * torch.eye(n, dtype=Hr.dtype)
    U = torch.linalg.cholesky(torch.cholesky_inverse(torch.linalg.cholesky(Hr)), upper=True)
    del U
    return time.perf_counter() - t0


def _qep_seconds(n, rows):
    """The QEP target of one stage (quantize.py:1330-1335, :1503): the ridge solve for M and W·M, torch fp64 on the
    CPU."""
    rng = np.random.default_rng(n + 1)
    A = torch.from_numpy(rng.standard_normal((n + 64, n)))
    H = A.T @ A / (n + 64)
    D = 0.01 * H
    W = torch.from_numpy(0.02 * rng.standard_normal((rows, n)))
    t0 = time.perf_counter()
    eye = torch.eye(n, dtype=H.dtype)
    M = eye + 0.5 * torch.linalg.solve(H + 0.1 * torch.diag(H).mean() * eye, D.T).T
    W @ M
    return time.perf_counter() - t0


CPU_SAMPLE_TOKENS = {2560: 16384, 4096: 8192, 9728: 2048}  # statistics sample per width (all tokens: ×48, ×96, ×384)


def _h_seconds_per_token(d):
    """The statistics GEMMs of one calibration token at width d: fp32 X_refᵀ(w⊙X) and Xᵀ(w⊙X) (quantize.py:1457-1470,
    torch on the CPU as the reference runs them), timed on CPU_SAMPLE_TOKENS[d] tokens."""
    from lookatmyquant_b200.workloads import stage_activations, token_weights
    nt = CPU_SAMPLE_TOKENS.get(d, 4096)
    x, xr = (t.float() for t in stage_activations(nt, d, seed=3000 + d, device="cpu"))
    w = token_weights(nt, seed=7, device="cpu").float()
    t0 = time.perf_counter()
    xw = x * w.reshape(-1, 1)
    xr.T @ xw
    x.T @ xw
    return (time.perf_counter() - t0) / nt


def _words_fit_at(d):
    from lookatmyquant_b200.layer import qwen3_4b_stages  # noqa: F401  (the widths come from the layer)
    values = np.fromfile(ROOT / "lookatmyquant_b200" / "tables" / "trellis_L12_k2_T256_s0_ema.f64", "<f8")
    _warm_oracle(values)
    W = 0.02 * np.random.default_rng(d).standard_normal((128, d))
    return words_fit(W, _dense_rotation(d), np.eye(d), np.zeros(d, dtype=bool), values)


def config3_components(stages=None):
    """The pieces of the reference's CPU path for one config-3 layer that the CPU baseline times, each a bounded
    sample: (key, function returning its measurement). A step of the reference arm times two of them."""
    from lookatmyquant_b200.layer import qwen3_4b_stages
    stages = stages or qwen3_4b_stages()
    widths = sorted({s.d for s in stages})
    comps = [(("h", d), (lambda d=d: _h_seconds_per_token(d))) for d in widths]
    comps += [(("fixed", d), (lambda d=d: _ldlq_call_fixed_seconds(d))) for d in widths]
    comps += [(("qep", s.name), (lambda s=s: _qep_seconds(s.d, sum(r for _, r in s.matrices)))) for s in stages]
    comps += [(("words", d), (lambda d=d: _words_fit_at(d))) for d in widths]
    return comps


def config3_total(meas: dict, tokens=384 * 2048, stages=None):
    """One layer's seconds from the components' measurements (each a list; the median is used), with every
    extrapolation factor stated:
    - statistics: seconds per token at each stage's width × the layer's tokens;
    - per ldlq_words call, the work it repeats whatever its rows (R·H·Rᵀ, the Environment) at the stage's width ×
      the calls (one per width group of every matrix, quantize.py:530-565);
    - the QEP target per stage (solve and W·M) at full size;
    - the word work (rotation, row scales, Viterbi sweep, dequantization) on the oracle port: a line fitted on 16 and
      128 rows per width, its per-call part × the calls and its per-row part × the layer's rows."""
    from lookatmyquant_b200.layer import qwen3_4b_stages
    stages = stages or qwen3_4b_stages()
    med = {k: (statistics.median(v) if not isinstance(v[0], tuple) else
               tuple(statistics.median(x[i] for x in v) for i in range(2))) for k, v in meas.items()}
    calls = {s.name: GROUPS_PER_MATRIX * len(s.matrices) for s in stages}
    h = sum(med[("h", s.d)] * tokens for s in stages)
    f = sum(calls[s.name] * med[("fixed", s.d)] for s in stages)
    q = sum(med[("qep", s.name)] for s in stages)
    w = sum(calls[s.name] * med[("words", s.d)][0] + sum(r for _, r in s.matrices) * med[("words", s.d)][1]
            for s in stages)
    widths = sorted({s.d for s in stages})
    desc = [f"H/D fp32 GEMMs {h:.0f} s (" + ", ".join(f"d={d}: {CPU_SAMPLE_TOKENS.get(d, 4096)} of {tokens} tokens, "
                                                      f"x{tokens / CPU_SAMPLE_TOKENS.get(d, 4096):.0f}" for d in widths) + ")",
            "R·H·Rᵀ + Environment per ldlq_words call at full width (" +
            ", ".join(f"{d}: {med[('fixed', d)]:.2f} s" for d in widths) + f") x{sum(calls.values())} calls: {f:.0f} s",
            f"QEP solve + W·M per stage at full size: {q:.0f} s",
            "row-trellis words fitted on 16 and 128 rows per width (" +
            ", ".join(f"d={d}: {med[('words', d)][0]:.2f} s/call + {med[('words', d)][1] * 1e3:.1f} ms/row"
                      for d in widths) + f") over the layer's {sum(r for s in stages for _, r in s.matrices)} rows: "
            f"{w:.0f} s"]
    return h + f + q + w, desc


def config3_cpu_sample(threads, tokens=384 * 2048, stages=None):
    """Every component timed once on this process's host threads (the repo arm's cpu_baseline leg)."""
    from oracle import core as O
    O.set_threads(threads)
    torch.set_num_threads(threads)
    meas = {k: [fn()] for k, fn in config3_components(stages)}
    v, desc = config3_total(meas, tokens, stages)
    return v, f"oracle port and torch on {threads} host threads, one layer extrapolated: " + "; ".join(desc)


WORKLOADS = {"config1": Config1, "config3": Config3}


def sweep_kernel_ms(wl, reps=3):
    """Average device time of the fused sweep kernel alone, on the stream it is launched on (CUDA events)."""
    from lookatmyquant_b200 import codes
    from lookatmyquant_b200.frame import Environment
    dev = wl.device
    R = codes.rht(wl.n, wl.in_seed).to(dev)
    X = wl.W @ R.T
    S = X.pow(2).mean(1).sqrt().clamp(min=1e-12)
    env = Environment(R @ wl.H @ R.T)
    codes._row_trellis_sweep(X, S, env, wl.code)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    total = 0.0
    for _ in range(reps):
        flush.zero_()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        codes._row_trellis_sweep(X, S, env, wl.code)
        e.record()
        e.synchronize()
        total += s.elapsed_time(e)
    return total / reps


def sweep_roofline(kms, algo_bytes, edges, pk):
    """The fused sweep is bound by FP32 issue (the trellis), so the ALU fraction is the binding one; the HBM fraction
    the north star asks for is reported as the `hbm` roofline."""
    achieved_gbs = algo_bytes / (kms * 1e-3) / 1e9
    sm_mhz = pk.get("sm_max_mhz", 1965.0)
    fp32_peak = SMS * FP32_LANES * sm_mhz * 1e6 / 1e12
    fp32_achieved = 3 * edges / (kms * 1e-3) / 1e12
    return {"kernel": "sweep_run_kernel (fused row-trellis LDLQ sweep)", "bound": "hbm", "achieved": achieved_gbs, "peak": pk["hbm_gbs"],
            "unit": "GB/s", "frac": achieved_gbs / pk["hbm_gbs"], "traffic": None, "kernel_ms": kms,
            "peak_source": pk["source"],
            "alu": {"achieved": fp32_achieved, "peak": fp32_peak, "unit": "T fp32 lane-ops/s",
                    "frac": fp32_achieved / fp32_peak, "note": "3 fp32 ops per trellis edge; the binding roofline"}}


PROBE_LAYERS = (0, 16, 31)  # the config-4 sample: every linear piece of a first, a middle and the last layer


def probe_sample(dev, rank, world, group):
    """BASELINE config 4 on a bounded sample: the KL probes (tr2, tr3, tr4) of every linear piece of PROBE_LAYERS of
    the 32-layer SmolLM2-360M-architecture model over 8 × 2048 held tokens, pieces split across the ranks; probes per
    hour = the sample's probes / the slowest rank's seconds in probes (a probe's cost falls with its layer, so the
    first, middle and last layers stand for the sweep's average)."""
    from lookatmyquant_b200 import measure
    torch.cuda.synchronize()
    res = measure.run(layers=PROBE_LAYERS, n_layers=32, windows=8, T=2048, device=dev, log=lambda s: None,
                      rank=rank, world=world, group=group)
    return {"probes_per_hour": res["probes per hour"], "probes": res["probes"],
            "seconds_in_probes": res["seconds in probes"], "layers": list(PROBE_LAYERS),
            "held_tokens": 8 * 2048, "options": ["tr2", "tr3", "tr4"], "kl_floor": res["kl floor"],
            "sweep": "224 pieces x 3 options = 672 probes", "piece": "TrellisLinear (trellis-dequant tensor-core GEMM)"}


def run_reference(args):
    """The reference arm: the reference's CPU path (its torch arithmetic, and the oracle port of its sweep) on all
    host threads. config3: every step times two of the layer's components (config3_components, in turn, each a
    bounded sample), and the value is one layer extrapolated from the median of each component's timed measurements
    (config3_total; the warm-up steps time every component once and are not used). config1: every step times the
    whole sample and the value is the median. ms_per_step is a step's wall time. Rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    from oracle import core as O
    O.set_threads(threads)
    torch.set_num_threads(threads)
    walls, sample = [], ""
    if args.workload == "config3":
        comps = config3_components()
        warm = {}
        for k, fn in comps:  # warm-up: every component once (not used)
            warm[k] = [fn()]
        meas = {}
        for i in range(args.steps):
            t0 = time.perf_counter()
            for j in (2 * i, 2 * i + 1):
                k, fn = comps[j % len(comps)]
                meas.setdefault(k, []).append(fn())
            walls.append(time.perf_counter() - t0)
        for k in warm:  # a component no timed step reached keeps its warm-up measurement
            meas.setdefault(k, warm[k])
        v, desc = config3_total(meas)
        counts = sorted({len(x) for x in meas.values()})
        sample = (f"oracle port and torch on {threads} host threads, one layer extrapolated from the median of "
                  f"{counts} timed samples per component: " + "; ".join(desc))
        spread = None
    else:
        times = []
        for i in range(args.warmup + args.steps):
            t0 = time.perf_counter()
            from lookatmyquant_b200.workloads import config1
            W, H, seed, in_seed = config1()
            values = np.fromfile(ROOT / "lookatmyquant_b200" / "tables" / "trellis_L12_k2_T256_s0_ema.f64", "<f8")
            x, sample = config1_cpu_sample(threads, W.numpy(), H.numpy(), in_seed, values)
            if i >= args.warmup:
                times.append(x)
                walls.append(time.perf_counter() - t0)
        v = statistics.median(times)
        spread = (max(times) - min(times)) / v if v else 0.0
    metric = Config3.metric if args.workload == "config3" else Config1.metric
    cfg = {"workload": args.workload}
    line = {"impl": "reference", "metric": metric, "value": v, "unit": "s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": statistics.mean(walls) * 1e3,
            "higher_is_better": False, "scaling": "strong" if args.workload == "config3" else "weak",
            "vs_baseline": None, "dtype": "f64+f32", "data": "synthetic (seeded)", "config": cfg,
            "value_is": "one layer (build) extrapolated from bounded CPU samples; ms_per_step is a step's wall time",
            "cpu_baseline": {"value": v, "unit": "s", "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": v, "unit": "s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    if spread is not None:
        line["step_spread"] = spread
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", default="config3", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-probes", action="store_true", help="skip the config-4 KL-probe sample")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        # NCCL prints its version banner (when NCCL_DEBUG is set) to file descriptor 1: point that descriptor at
        # stderr and keep Python's stdout on the original one, so stdout carries only the JSON line
        sys.stdout.flush()
        sys.stdout = os.fdopen(os.dup(1), "w", buffering=1)
        os.dup2(2, 1)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=dev)
    from lookatmyquant_b200 import _lib
    _lib.load()
    group = torch.distributed.group.WORLD if world > 1 else None
    wl = WORKLOADS[args.workload](dev) if args.workload == "config1" else WORKLOADS[args.workload](dev, group=group)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)  # 256 MB > 126 MB L2
    for _ in range(max(args.warmup, 3)):
        wl.step()
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    barrier()
    launches0 = _lib.kernel_launches()
    with Clocks(local) as clk:
        for i in range(args.steps):
            flush.zero_()
            starts[i].record()
            wl.step(timed=True) if hasattr(wl, "stage_ms") else wl.step()
            ends[i].record()
        barrier()
        ms = sum(s_.elapsed_time(e_) for s_, e_ in zip(starts, ends)) / args.steps
    launches = (_lib.kernel_launches() - launches0) // args.steps
    # e2e: the same build through the public API from pinned host memory, result read back, every step
    wl.prepare_e2e()
    wl.e2e_step()  # untimed warm-up: the first call's device allocations and pinned read-back buffers
    barrier()
    e2e_ms = []
    for i in range(min(args.steps, 3)):
        flush.zero_()
        barrier()
        t0 = time.perf_counter()
        wl.e2e_step()
        barrier()
        e2e_ms.append((time.perf_counter() - t0) * 1e3)
    t = torch.tensor([ms, statistics.mean(e2e_ms)], device=dev, dtype=torch.float64)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms, e2e = float(t[0]), float(t[1])
    pk = peaks()
    roof = wl.roofline(pk)
    h2d, d2h = wl.e2e_bytes()
    cfg = wl.config()
    cfg["l2"] = cfg.get("l2", "flushed (256 MB write) before every step")
    line = {
        "metric": wl.metric, "value": ms / 1e3, "unit": "s", "n_gpus": world, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": ms, "higher_is_better": False,
        "scaling": "strong" if wl.name == "config3" else "weak", "vs_baseline": None, "dtype": "bf16+f64+f32",
        "data": "synthetic (seeded; no dataset or checkpoint)", "config": cfg,
        "e2e": {"value": e2e / 1e3, "unit": "s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "roofline": roof, "gpu_launches": launches, "clocks": clk.summary(),
    }
    if getattr(wl, "h_accum", None):
        # the metric's "H-accum TFLOP/s": config 2 is this statistics pass (786,432 weighted tokens; d = 2560 is the
        # q/k/v and gate/up stages' input, d = 9728 the down_proj stage's), H and D, on each rank's token shard
        line["h_accum_tflops"] = {k: {"d": v["d"], "tokens_per_rank": v["tokens"], "ms": round(v["ms"], 2),
                                      "tflops": round(v["tflops_2Nd2"] * world, 1)} for k, v in wl.h_accum.items()}
    if args.workload == "config3" and not args.no_probes:
        line["config4"] = probe_sample(dev, rank, world, group)
    if getattr(wl, "stage_ms", None):
        # per-stage device time of the timed steps (this rank's; the step's all-gather of states is outside them)
        line["stage_ms"] = {k: round(statistics.mean(a.elapsed_time(b) for a, b in v), 2)
                            for k, v in wl.stage_ms.items()}
    if rank == 0 and not args.no_cpu_baseline:
        v, sample = wl.cpu_sample(os.cpu_count() or 1)
        line["cpu_baseline"] = {"value": v, "unit": "s", "cores": os.cpu_count() or 1, "kind": "port",
                                "sample": sample}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
