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

    def cpu_sample(self, threads):
        """The oracle on the first 256 rows (a tenth of the matrix; rows are independent, so time scales with rows)."""
        from oracle import core as O
        O.set_threads(threads)
        rows = 256
        W = self.W_host[:rows].numpy()
        t0 = time.perf_counter()
        O.ldlq_row_words(W, self.H_host.numpy(), self.code.values.numpy(), 12, 2, self.in_seed)
        dt = time.perf_counter() - t0
        return dt * self.m / rows, f"oracle ldlq_row_words on 256 of 2560 rows, scaled x{self.m / rows:g}"


WORKLOADS = {"config1": Config1}


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


def run_reference(args):
    """The reference arm: the CPU oracle port of the reference's path, all host threads, bounded sample per step."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    from lookatmyquant_b200.workloads import config1
    from oracle import core as O
    O.set_threads(threads)
    W, H, seed, in_seed = config1()
    values = np.fromfile(ROOT / "lookatmyquant_b200" / "tables" / "trellis_L12_k2_T256_s0_ema.f64", dtype="<f8")
    rows = 256
    times = []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        O.ldlq_row_words(W[:rows].numpy(), H.numpy(), values, 12, 2, in_seed)
        if i >= args.warmup:
            times.append((time.perf_counter() - t0) * W.shape[0] / rows)
    v = statistics.mean(times)
    sample = f"oracle ldlq_row_words on 256 of 2560 rows per step, scaled x{W.shape[0] / rows:g}"
    print(json.dumps({"impl": "reference", "metric": Config1.metric, "value": v, "unit": "s", "n_gpus": args.gpus,
                      "steps": args.steps, "warmup": args.warmup, "ms_per_step": v * 1e3, "higher_is_better": False,
                      "scaling": "weak", "vs_baseline": None, "dtype": "f64+f32", "data": "synthetic",
                      "config": {"workload": "config1", "rows": 2560, "cols": 960, "bits": 2},
                      "cpu_baseline": {"value": v, "unit": "s", "cores": threads, "kind": "port", "sample": sample},
                      "e2e": {"value": v, "unit": "s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", default="config1", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
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
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=dev)
    from lookatmyquant_b200 import _lib
    _lib.load()
    wl = WORKLOADS[args.workload](dev)
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
    launches0 = _lib.LAUNCHES["count"]
    with Clocks(local) as clk:
        for i in range(args.steps):
            flush.zero_()
            starts[i].record()
            wl.step()
            ends[i].record()
        barrier()
        ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends)) / args.steps
        # e2e: the same build through the public API from pinned host memory, result read back, every step
        e2e_ms = []
        for i in range(args.steps):
            flush.zero_()
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            wl.e2e_step()
            torch.cuda.synchronize()
            e2e_ms.append((time.perf_counter() - t0) * 1e3)
    launches = _lib.LAUNCHES["count"] - launches0
    t = torch.tensor([ms, statistics.mean(e2e_ms)], device=dev, dtype=torch.float64)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms, e2e = float(t[0]), float(t[1])
    kms = sweep_kernel_ms(wl)
    pk = peaks()
    algo_bytes, edges = wl.sweep_algorithmic()
    achieved_gbs = algo_bytes / (kms * 1e-3) / 1e9
    sm_mhz = pk.get("sm_max_mhz", 1965.0)
    fp32_peak = SMS * FP32_LANES * sm_mhz * 1e6 / 1e12  # T lane-ops/s at the max SM clock
    fp32_achieved = 3 * edges / (kms * 1e-3) / 1e12  # sub, mul, add per trellis edge
    h2d, d2h = wl.e2e_bytes()
    line = {
        "metric": wl.metric, "value": ms / 1e3, "unit": "s", "n_gpus": world, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": ms, "higher_is_better": False, "scaling": "weak",
        "vs_baseline": None, "dtype": "f64+f32", "data": "synthetic",
        "config": {"workload": wl.name, "rows": wl.m, "cols": wl.n, "bits": 2, "trellis": "L=12 k=2 (reference table)",
                   "width": 16, "look": 8, "lazy": 128, "l2": "flushed (256 MB write) before every step"},
        "e2e": {"value": e2e / 1e3, "unit": "s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "roofline": {"kernel": "sweep_rowtrellis_kernel", "bound": "hbm", "achieved": achieved_gbs,
                     "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": achieved_gbs / pk["hbm_gbs"], "traffic": None,
                     "kernel_ms": kms, "peak_source": pk["source"],
                     "alu": {"achieved": fp32_achieved, "peak": fp32_peak, "unit": "T fp32 lane-ops/s",
                             "frac": fp32_achieved / fp32_peak, "note": "3 fp32 ops per trellis edge; binding roofline"}},
        "gpu_launches": launches,
        "clocks": clk.summary(),
    }
    if rank == 0 and not args.no_cpu_baseline:
        v, sample = wl.cpu_sample(os.cpu_count() or 1)
        line["cpu_baseline"] = {"value": v, "unit": "s", "cores": os.cpu_count() or 1, "kind": "port",
                                "sample": sample}
    if rank == 0:
        print(json.dumps(line))
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
