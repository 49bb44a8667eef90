"""Row-plan build of one decoder layer on B200: the lm2 build's per-layer work (quantize.py `quantize_stage`).

Reference (ShinMegamiBoson/lookatmyquant), per stage of matrices that read one input (quantize.py:1404-1568):

  1. H = Σ_t w_t x_t x_tᵀ / n_tok and the QEP moment D = Σ_t w_t x_ref,t x_tᵀ / n_tok − H  (:1412-1470)
  2. M = I + α·(solve(H + λ·mean(diag H)·I, Dᵀ))ᵀ, target = W·M                              (:1330-1335, :1503)
  3. per row group of the row plan, word('tr{b}x', target[rows], H, seed, in_seed, out_rot=False) (:530-565, :1531):
     X = target·R_inᵀ, S = row RMS, Hr = R_in·H·R_inᵀ, U from Environment(Hr), the row-trellis LDLQ sweep
     (codes.py:413-462), W_q = diag(S)·V[states]·R_in.

Row groups are swept by one kernel for the whole stage (rows never interact under Refit; each row carries its own
width k), the rotation is factored (rotation.py), H and D come from the tcgen05 kernel (hessian.py). With a process
group, tokens are sharded for H and D (the fp32 accumulators are summed with one all-reduce per stage) and rows are
sharded for the sweep (states and scales gathered at the end).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch

from . import codes
from .codes import LAZY, stacked_tables
from .frame import Environment
from .hessian import Statistics
from .linalg import CrossTarget, cholesky_inverse_lower, ridge, status_check
from .rotation import Rotation

ALPHA, LAM = 0.5, 0.1  # QEP strength of the lm2 build (--cross-alpha 0.5) and the ridge (quantize.py:93)


@dataclass
class StageSpec:
    name: str
    d: int
    matrices: list  # (name, rows)
    block: str      # "self_attn" or "mlp": the Hadamard seed block (compiler_arch.block_seed)


def qwen3_4b_stages(hidden=2560, heads=32, kv_heads=8, head_dim=128, mlp=9728):
    """The four stages of a Qwen3-4B-class decoder layer (quantize.py STAGES, :89-91)."""
    return [StageSpec("attn_in", hidden, [("self_attn.q_proj", heads * head_dim), ("self_attn.k_proj", kv_heads * head_dim),
                                          ("self_attn.v_proj", kv_heads * head_dim)], "self_attn"),
            StageSpec("o_in", heads * head_dim, [("self_attn.o_proj", hidden)], "self_attn"),
            StageSpec("mlp_in", hidden, [("mlp.gate_proj", mlp), ("mlp.up_proj", mlp)], "mlp"),
            StageSpec("down_in", mlp, [("mlp.down_proj", hidden)], "mlp")]


def row_plan(rows: int, seed: int, group: int = 64, widths=(1, 2, 3, 4), probs=(0.15, 0.45, 0.30, 0.10)) -> torch.Tensor:
    """Per-row bit widths drawn per group of `group` rows (config 3's synthetic plan; rowgroup_alloc plans use runs of
    64 rows)."""
    g = torch.Generator().manual_seed(seed)
    choice = torch.multinomial(torch.tensor(probs, dtype=torch.float64), (rows + group - 1) // group, replacement=True,
                               generator=g)
    return torch.tensor(widths, dtype=torch.uint8)[choice].repeat_interleave(group)[:rows]


_SIDE = {}
_FACTOR = {}


def _side_stream(dev) -> torch.cuda.Stream:
    """The stage's QEP stream, at high priority: its factorization and the targets it feeds run first, the
    environment's factorization (whose leaf steps leave most SMs idle) fills in around them."""
    if dev not in _SIDE:
        _SIDE[dev] = torch.cuda.Stream(device=dev, priority=-1)
    return _SIDE[dev]


def row_shard(total: int, rank: int, world: int, group: int = 64) -> tuple[int, int]:
    """Rows [r0, r1) of a stage that `rank` sweeps: whole runs of `group` rows, split as evenly as possible."""
    groups = (total + group - 1) // group
    g0, g1 = groups * rank // world, groups * (rank + 1) // world
    return g0 * group, min(total, g1 * group)


def cross_target(H: torch.Tensor, D: torch.Tensor, alpha: float = ALPHA, lam: float = LAM) -> torch.Tensor:
    """M = I + α·(solve(H + λ·mean(diag H)·I, Dᵀ))ᵀ (quantize.py:1330-1335), fp64 on H's device (tensor cores)."""
    return CrossTarget(H, D, alpha, lam).M


@dataclass
class StageResult:
    states: dict = field(default_factory=dict)   # matrix name -> rows × n int16 (this rank's rows)
    scales: dict = field(default_factory=dict)   # matrix name -> rows fp64
    Wq: dict = field(default_factory=dict)       # matrix name -> rows × n fp64 (dequantized)
    row_range: dict = field(default_factory=dict)


def build_stage(spec: StageSpec, weights: dict, x: torch.Tensor, x_ref: torch.Tensor, w: torch.Tensor | None,
                bits: dict, layer: int = 0, group=None, dequantize: bool = True, tables=None,
                n_tok_total: int | None = None) -> StageResult:
    """One stage: statistics, QEP target, rotation, environment and the fused row-trellis sweep over every row of the
    stage's matrices. `weights[name]` is rows × d (any float dtype, on the device), `bits[name]` the per-row widths.
    With a process group, x/x_ref/w are this rank's token shard and each rank sweeps a contiguous share of rows."""
    st = Statistics(spec.d, cross=True, device=x.device)
    st.add(x, w, x_ref)
    return build_stage_from_statistics(spec, weights, st, bits, layer, group, dequantize, tables, n_tok_total)


def _in_seed(spec: StageSpec, layer: int) -> int:
    """The stage's input-rotation seed (quantize.py:1531: 1000·layer + 100·block_seed + 1)."""
    return 1000 * layer + 100 * {"self_attn": 2, "mlp": 3}[spec.block] + 1


def _reduce_finalize(st: Statistics, group, n_tok_total):
    """H and D of a stage: the ranks' fp32 accumulators summed (one all-reduce each), then finalized."""
    n_tok = st.n_tok
    if group is not None:
        torch.distributed.all_reduce(st.accH, group=group)
        torch.distributed.all_reduce(st.accD, group=group)
        if n_tok_total is None:  # ranks may hold unequal shares (token_shard splits whole chunks): sum them
            # a fill on the device, not a copy from host memory (which would queue behind a host build's bulk copies)
            cnt = torch.full((1,), float(n_tok), dtype=torch.float64, device=st.accH.device)
            torch.distributed.all_reduce(cnt, group=group)
            n_tok_total = int(cnt.item())
        n_tok = n_tok_total
    return st.finalize(n_tok)


def build_stage_from_statistics(spec: StageSpec, weights: dict, st: Statistics, bits: dict, layer: int = 0, group=None,
                                dequantize: bool = True, tables=None, n_tok_total: int | None = None, HD=None,
                                factors=None, rot=None) -> StageResult:
    """The stage after its statistics have been accumulated (all of this rank's tokens added to `st`). `HD` (H, D)
    and `factors` (env, Linv, qep_status) skip the reduction and the factorizations when they were done already
    (build_stages_sharded); `rot` is the stage's input rotation when the caller made it already."""
    dev = st.device if st is not None else HD[0].device
    world = group.size() if group is not None else 1
    rank = group.rank() if group is not None else 0
    H, D = _reduce_finalize(st, group, n_tok_total) if HD is None else HD
    in_seed = _in_seed(spec, layer)
    # all rows of the stage, this rank's contiguous share (whole 64-row groups)
    names = [nm for nm, _ in spec.matrices]
    total = sum(r for _, r in spec.matrices)
    r0, r1 = row_shard(total, rank, world)
    # the QEP map (a factorization of H + λμI) with the rotated targets it feeds, and the environment (a
    # factorization of R·H·Rᵀ), are independent: the first runs on a side stream while the second runs on the main one
    main = torch.cuda.current_stream(dev)
    side = _side_stream(dev)
    rot = Rotation(spec.d, in_seed, dev) if rot is None else rot
    if factors is None and world >= 2:
        # two ranks factor at once, one matrix each, and broadcast the factors (NVLink): the QEP's inverse Cholesky
        # factor from rank 1, the environment's U from rank 0
        factors = _factors_on_two_ranks(rot, H, rank, group)
    side.wait_stream(main)
    Xs, ks, spans, off = [], [], {}, 0
    with torch.cuda.stream(side):
        if factors is None:
            qep = CrossTarget(H, D, ALPHA, LAM, rows=r1 - r0)
        else:
            qep = CrossTarget(None, D, ALPHA, LAM, rows=r1 - r0, Linv=factors[1], check=status_check(factors[2]))
        for nm, rows in spec.matrices:
            a, b = max(r0, off), min(r1, off + rows)
            if a < b:
                target = qep.apply(weights[nm][a - off:b - off].to(torch.float64))
                Xs.append(rot.rows(target))
                ks.append(bits[nm][a - off:b - off])
                spans[nm] = (a - off, b - off)
            off += rows
    env = Environment(rot.conj(H)) if factors is None else factors[0]
    main.wait_stream(side)
    qep.record_stream(main)
    for t in Xs:
        t.record_stream(main)
    res = StageResult(row_range=spans)
    if not Xs:
        return res
    X = torch.cat(Xs) if len(Xs) > 1 else Xs[0]
    row_bits = torch.cat(ks).to(dev, torch.uint8) if len(ks) > 1 else ks[0].to(dev, torch.uint8)
    S = X.pow(2).mean(1).sqrt().clamp(min=1e-12)
    states, settled = sweep_rows(X, S, env, row_bits, tables)
    o = 0
    for nm in names:
        if nm not in spans:
            continue
        a, b = spans[nm]
        res.states[nm] = states[o:o + b - a]
        res.scales[nm] = S[o:o + b - a]
        if dequantize:
            res.Wq[nm] = rot.rows_t(settled[o:o + b - a] * S[o:o + b - a, None])
        o += b - a
    env.check()
    qep.check()
    return res


def _factor_stream(dev) -> torch.cuda.Stream:
    if dev not in _FACTOR:
        _FACTOR[dev] = torch.cuda.Stream(device=dev)
    return _FACTOR[dev]


def build_stages_sharded(stages, weights: dict, stats: list, bits: dict, layer: int = 0, group=None,
                         dequantize: bool = True, tables=None, n_tok_total: int | None = None) -> dict:
    """All stages of a layer over a group of 2 or more ranks, from their accumulated statistics: every stage's H and D
    reduced first, then every stage's two factorizations queued at once on the rank pairs `factor_owners` assigns
    (with 8 ranks each stage has its own pair) on a factorization stream, then stage by stage — the smallest first —
    the factors are broadcast as soon as that stage's are done and each rank maps and sweeps its rows. The
    factorizations of different stages overlap one another, and a rank that owns the large stage's factorization
    sweeps the smaller stages' rows while it runs; the results equal build_stage's. Returns {stage: StageResult}
    (this rank's rows)."""
    world, rank = group.size(), group.rank()
    HD = [_reduce_finalize(st, group, n_tok_total) for st in stats]
    owners = factor_owners([s.d for s in stages], world)
    dev = HD[0][0].device
    rots = [Rotation(s.d, _in_seed(s, layer), dev) for s in stages]
    order = sorted(range(len(stages)), key=lambda i: (stages[i].d, i))  # the same on every rank
    main, fs = torch.cuda.current_stream(dev), _factor_stream(dev)
    fs.wait_stream(main)
    bufs, done = [None] * len(stages), [None] * len(stages)
    with torch.cuda.stream(fs):
        for i in order:
            bufs[i] = _own_factors(rots[i], HD[i][0], rank, *owners[i])
            done[i] = torch.cuda.Event()
            done[i].record(fs)
    for b in bufs:
        for t in b:
            t.record_stream(main)
    out = {}
    for i in order:
        s = stages[i]
        main.wait_event(done[i])
        factors = _share_factors(rots[i], HD[i][0], bufs[i], *owners[i], group)
        out[s.name] = build_stage_from_statistics(s, weights, None, bits, layer, group, dequantize, tables,
                                                  n_tok_total, HD=HD[i], factors=factors, rot=rots[i])
    return {s.name: out[s.name] for s in stages}


def _own_factors(rot, H, rank: int, env_rank: int, qep_rank: int):
    """Queues this rank's share of a stage's two factorizations — Environment(R·H·Rᵀ) on `env_rank`, the QEP's inverse
    Cholesky factor of H + λ·mean(diag H)·I on `qep_rank` — and returns the buffers the owners broadcast (empty ones to
    receive into elsewhere): (Linv, qep_status, U, dead, env_status)."""
    n, dev = H.shape[0], H.device
    qst = torch.zeros(1, dtype=torch.int32, device=dev)
    est = torch.zeros(1, dtype=torch.int32, device=dev)
    if rank == qep_rank:
        Linv = cholesky_inverse_lower(ridge(H, LAM), deferred=True, status=qst)[0]
    else:
        Linv = torch.empty(n, n, dtype=torch.float64, device=dev)
    if rank == env_rank:
        env0 = Environment(rot.conj(H), status=est)
        U, dead = env0.U, env0.dead.to(torch.uint8)
    else:
        U = torch.empty(n, n, dtype=torch.float64, device=dev)
        dead = torch.empty(n, dtype=torch.uint8, device=dev)
    return Linv, qst, U, dead, est


def _share_factors(rot, H, bufs, env_rank: int, qep_rank: int, group):
    """Broadcasts a stage's factors from their owners (NVLink) and returns (env, Linv, qep_status) on every rank."""
    Linv, qst, U, dead, est = bufs
    src_q = torch.distributed.get_global_rank(group, qep_rank)
    src_e = torch.distributed.get_global_rank(group, env_rank)
    torch.distributed.broadcast(Linv, src=src_q, group=group)
    torch.distributed.broadcast(qst, src=src_q, group=group)
    torch.distributed.broadcast(U, src=src_e, group=group)
    torch.distributed.broadcast(dead, src=src_e, group=group)
    torch.distributed.broadcast(est, src=src_e, group=group)
    return Environment.from_factor(lambda: rot.conj(H), U, dead, est), Linv, qst


def _factors_on_two_ranks(rot, H, rank: int, group):
    """The stage's two factorizations on two ranks at once — Environment(R·H·Rᵀ) on rank 0, the QEP's inverse
    Cholesky factor of H + λ·mean(diag H)·I on rank 1 — each queued before any collective, then broadcast to the
    group (NVLink) with their status words. Returns (env, Linv, qep_status) on every rank."""
    return _share_factors(rot, H, _own_factors(rot, H, rank, 0, 1), 0, 1, group)


def factor_owners(dims, world: int) -> list:
    """(env_rank, qep_rank) per stage: the stages' factorizations spread over the group's rank pairs, the largest
    first onto the least loaded pair (cost ∝ d³), so with 8 ranks each stage of a layer has its own pair."""
    pairs = max(1, world // 2)
    load = [0.0] * pairs
    owners = [None] * len(dims)
    for i in sorted(range(len(dims)), key=lambda i: -dims[i]):
        p = min(range(pairs), key=lambda q: load[q])
        load[p] += float(dims[i]) ** 3
        owners[i] = (2 * p, 2 * p + 1) if world >= 2 else (0, 0)
    return owners


_COPY = {}


def _weight_groups(w_host: torch.Tensor, dev):
    """The weighted tokens of a chunk, found on the host: [(device int32 indices, w), ...] per distinct weight when
    there are few (Statistics gathers each group and adds it once, scaled by w − 1), else the indices of all of them
    (the hi/lo split). The copies to the device are queued on the current stream."""
    from .hessian import MAX_WEIGHT_GROUPS
    idx = torch.nonzero(w_host != 1.0).flatten().to(torch.int32)
    vals = torch.unique(w_host[idx.long()]).tolist() if idx.numel() else []
    if len(vals) > MAX_WEIGHT_GROUPS:
        return idx.pin_memory().to(dev, non_blocking=True)
    out = []
    for v in vals:
        sel = idx if len(vals) == 1 else idx[w_host[idx.long()] == v]
        out.append((sel.contiguous().pin_memory().to(dev, non_blocking=True), float(v)))
    return out


def _copy_stream(dev) -> torch.cuda.Stream:
    if dev not in _COPY:
        _COPY[dev] = torch.cuda.Stream(device=dev)
    return _COPY[dev]


def tail_order(stages, world: int = 1) -> list:
    """The stages ordered by the work that follows their statistics, largest first: the two factorizations (∝ d³)
    and the sweep of this rank's rows (∝ rows·d / world). A host build copies the stages in this order, so the stage
    whose factor-and-sweep tail is shortest arrives last and little compute is left once the last byte is resident.
    The coefficients are B200 timings (d = 9728: ~130 ms of factorizations and QEP map; 2560 x 9728 rows swept in
    ~74 ms); only the order matters."""
    def tail(s):
        rows = sum(r for _, r in s.matrices)
        return 1.4e-13 * float(s.d) ** 3 + 2.5e-9 * rows * s.d / max(1, world)
    return sorted(stages, key=lambda s: -tail(s))


def build_layer_from_host(stages, weights, acts, w, bits, layer: int = 0, group=None, n_tok_total: int | None = None,
                          chunk_tokens: int = 65536, device=None):
    """The layer build from host memory: `weights[name]` and `acts[stage] = (x, x_ref)` are pinned CPU tensors (this
    rank's token shard), `w` the pinned per-token weights. Every copy is queued at once on a copy stream, chunk by
    chunk and stage by stage, so the statistics kernel consumes each chunk as soon as it is resident and the later
    stages' activations arrive while the earlier stages factor and sweep: the build takes about the longer of the
    host→device transfer and the compute instead of their sum. The stages go in `tail_order` (each stage's inputs are
    given, so the order changes no result): the stage with the least work after its statistics comes last. The
    weighted tokens of each chunk are found on the host. Everything small the stages need from the host (the row
    widths, the rotations' signs and factors) goes to the device before the bulk copies are queued: a copy from
    pageable memory queued behind them would wait for all of them. Returns {stage: StageResult} with states and
    scales in pinned host memory (the call synchronizes)."""
    dev = torch.device(device or "cuda")
    copy, main = _copy_stream(dev), torch.cuda.current_stream(dev)
    tables = stacked_tables(12, 256, dev)
    stages = tail_order(stages, group.size() if group is not None else 1)
    bits = {nm: bits[nm].to(dev) for s in stages for nm, _ in s.matrices}
    rots = {s.name: Rotation(s.d, _in_seed(s, layer), dev) for s in stages}
    copy.wait_stream(main)
    staged = []
    with torch.cuda.stream(copy):
        w_d = w.to(dev, non_blocking=True)
        for s in stages:
            x_h, xr_h = acts[s.name]
            wts = {nm: weights[nm].to(dev, non_blocking=True) for nm, _ in s.matrices}
            x_d = torch.empty(x_h.shape, dtype=x_h.dtype, device=dev)
            xr_d = torch.empty(xr_h.shape, dtype=xr_h.dtype, device=dev)
            chunks = []
            for c0 in range(0, x_h.shape[0], chunk_tokens):
                c1 = min(c0 + chunk_tokens, x_h.shape[0])
                idx = _weight_groups(w[c0:c1], dev)
                x_d[c0:c1].copy_(x_h[c0:c1], non_blocking=True)
                xr_d[c0:c1].copy_(xr_h[c0:c1], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(copy)
                chunks.append((c0, c1, idx, ev))
            staged.append((x_d, xr_d, wts, chunks))
    def group_tensors(g):
        return [g] if isinstance(g, torch.Tensor) else [t for t, _ in g]
    for t in [w_d] + [t for x_d, xr_d, wts, chunks in staged
                      for t in [x_d, xr_d, *wts.values(), *(u for c in chunks for u in group_tensors(c[2]))]]:
        t.record_stream(main)
    out = {}
    for i, s in enumerate(stages):
        x_d, xr_d, wts, chunks = staged[i]
        staged[i] = None  # the stage's activations are freed once its statistics are done
        st = Statistics(s.d, cross=True, device=dev)
        for c0, c1, idx, ev in chunks:
            main.wait_event(ev)
            st.add(x_d[c0:c1], w_d[c0:c1], xr_d[c0:c1], weighted=idx)
        del x_d, xr_d, chunks
        res = build_stage_from_statistics(s, wts, st, bits, layer, group, False, tables, n_tok_total,
                                          rot=rots[s.name])
        for nm in list(res.states):
            res.states[nm] = res.states[nm].to("cpu", non_blocking=True)
            res.scales[nm] = res.scales[nm].to("cpu", non_blocking=True)
        out[s.name] = res
    torch.cuda.synchronize(dev)
    return out


def sweep_rows(X, S, env, row_bits, tables=None):
    """The fused row-trellis LDLQ sweep (lamq_ldlq_rowtrellis) with per-row widths; returns (states, settled).
    `tables` may instead be {width: (L, values)} codebooks with L < 12 (BASELINE config 3's synthetic codebooks):
    then each width's rows take the generic sweep with the small-state Viterbi (codes.generic_trellis_sweep)."""
    if isinstance(tables, dict):
        dev = X.device
        states = torch.empty(X.shape, dtype=torch.int16, device=dev)
        settled = torch.empty_like(X)
        for k, (L, values) in tables.items():
            idx = torch.nonzero(row_bits.to(dev) == k).flatten()
            if idx.numel() == 0:
                continue
            code = codes.RowTrellisCode(L, k, T=256, width=codes.WIDTH, look=codes.LOOK, values=values)
            st, se = codes.generic_trellis_sweep(X[idx].contiguous(), S[idx].contiguous(), env, code)
            states[idx], settled[idx] = st, se
        return states, settled
    from . import _lib
    from ._lib import check, ptr, stream_ptr
    dev = X.device
    rows, n = X.shape
    T = X.contiguous().clone()
    states = torch.empty(rows, n, dtype=torch.int16, device=dev)
    settled = torch.empty(rows, n, dtype=torch.float64, device=dev)
    tables = stacked_tables(12, 256, dev) if tables is None else tables
    dead = env.dead.to(dev, torch.uint8) if bool(env.dead.any()) else None
    ws = torch.empty(_lib.load().lamq_ldlq_rowtrellis_workspace_size(rows, n), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        check(_lib.load().lamq_ldlq_rowtrellis(
            ptr(T), n, rows, n, ptr(env.U), env.U.stride(0), ptr(dead), ptr(S.contiguous()), ptr(tables),
            ptr(row_bits), 0, 12, codes.WIDTH, codes.LOOK, LAZY, ptr(states), ptr(settled), ptr(ws), ws.numel(),
            stream_ptr(dev)),
            "lamq_ldlq_rowtrellis")
    return states, settled


def build_layer(stages, weights, acts, w, bits, layer: int = 0, group=None, dequantize: bool = True,
                n_tok_total: int | None = None):
    """All stages in order (true-sequential within the layer). `acts[stage] = (x, x_ref)`. Returns {stage: result}."""
    tables = stacked_tables(12, 256, acts[stages[0].name][0].device)
    return {s.name: build_stage(s, weights, *acts[s.name], w, bits, layer, group, dequantize, tables, n_tok_total)
            for s in stages}


def main():
    """Builds one synthetic config-3 layer (the benchmark's workload) once and prints per-stage timings: the command
    the per-kernel launch lists in profiles/ were captured with."""
    import argparse
    import json
    import time
    from .workloads import config3
    ap = argparse.ArgumentParser(description=main.__doc__)
    ap.add_argument("--tokens", type=int, default=384 * 2048)
    ap.add_argument("--repeat", type=int, default=1)
    ap.add_argument("--codebooks", choices=["reference", "synthetic"], default="reference",
                    help="the reference's 4096-state L = 12 tables for every width, or BASELINE config 3's "
                         "2^(bits+4)-entry Lloyd-Max codebooks (L = bits + 4, the generic sweep)")
    a = ap.parse_args()
    dev = torch.device("cuda")
    stages, weights, acts, w, bits = config3(a.tokens, device=dev)
    tables = stacked_tables(12, 256, dev) if a.codebooks == "reference" else \
        {b: codes.synthetic_codebook(b) for b in (1, 2, 3, 4)}
    for _ in range(a.repeat):
        times = {}
        for s in stages:
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            build_stage(s, weights, *acts[s.name], w, bits, 0, None, True, tables)
            torch.cuda.synchronize()
            times[s.name] = round((time.perf_counter() - t0) * 1e3, 2)
        print(json.dumps({"codebooks": a.codebooks, "stage_ms": times, "total_ms": round(sum(times.values()), 2)}),
              flush=True)


if __name__ == "__main__":
    main()
