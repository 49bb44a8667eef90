// The block-LDLQ sweep with a row trellis (the lm2 build's per-matrix loop).
//
// Reference: opgraph/syntax.py:86-124 (`sweep`), with the projection of opgraph/codes.py:442-450 and
// RowTrellisCode.step (codes.py:397-404). Rows never interact under Refit (codes.py:417-418), so inside a run of
// `lazy` columns every row is independent; across runs, the run's errors reach all later columns of all rows through
// one matrix product. The sweep is therefore a sequence of runs, each two launches:
//
//   sweep_run_kernel — a persistent grid of 8 warp pairs per CTA (trellis_pair.cuh: 64 states per thread, fp32x2
//     arithmetic); each pair takes rows one at a time — the first round spread over the CTAs (row i of the list to CTA
//     i mod grid), then from a per-run counter — from a list grouped by width, widest first, so the SMs stay evenly
//     loaded whether a stage has 300 rows per GPU or 20,000. Per row the run's targets plus the `look` columns after
//     it go to the pair's slot in shared memory (Trun); per block of `width` columns the pair decodes the block plus
//     `look` columns ahead (in units of the row scale, from the row's last state; the look-ahead past the run is stale
//     by design, as in the reference), settles the block with the fp64 table values, writes the columns as they stood
//     to T (what sweep returns), solves z·U_BB = E by substitution, keeps z in the block's Trun slots and updates the
//     rest of the run in shared memory (syntax.py:117-120); at the end of the run the row's z go to Z and its last
//     state to a per-row array for the next run;
//   lamq_dgemm — T[:, b1:] −= Z·U[b0:b1, b1:] for all rows at once (syntax.py:122-123), on the fp64 tensor cores,
//     each U element read once per 128 rows instead of once per tile.
#include <algorithm>

#include "lamq_common.cuh"
#include "trellis_pair.cuh"
#include "trellis_warp.cuh"

namespace lamq {

namespace {

constexpr int kWarps = 16;
constexpr int kPairs = kWarps / 2;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxWin = 24;  // RowTrellisCode windows: width 16 + look 8
constexpr int kMaxLazy = 128;

struct SweepParams {
    double *T;
    int64_t ldT;
    int n;
    const int32_t *rowlist;   // row indices grouped by width (widest first)
    const int *nrows;         // device: rows in the list
    int *counters;            // device: per run, rows taken after the first, spread round
    const uint8_t *row_bits;  // per-row width or null
    int k_all;
    const double *U;
    int64_t ldU;
    const uint8_t *dead;
    const double *S;
    const double *tables;
    int width, look, lazy;
    int trun_stride;          // doubles per Trun row
    double *Z;                // rows x kMaxLazy: each row's z over the run (the run product's left factor)
    int *rstate;              // rows: each row's last state after the runs so far
    int b0, b1, run;          // this launch's run [b0, b1)
    int16_t *states;
    double *settled;
};

// Per-pair Viterbi scratch, carved per width: two best buffers of R floats and kMaxWin steps of back-pointers (WORDS x
// 64 words each) — at most 22 KiB (k = 1) — and 8 words for the final reduction.
template <int K>
constexpr size_t pair_bytes() {
    return 2 * (size_t)PairTrellis<K>::R * sizeof(float) + (size_t)kMaxWin * 64 * PairTrellis<K>::WORDS * sizeof(uint32_t);
}
constexpr size_t kPairMax = pair_bytes<1>() > pair_bytes<2>() ? pair_bytes<1>() : pair_bytes<2>();
constexpr size_t kPairViterbiBytes = kPairMax + 8 * sizeof(float);
constexpr size_t kUnionBytes = kPairs * kPairViterbiBytes;

// One row's run by the warp pair: tr is the pair's Trun slot, wv its Viterbi scratch, st_slot a shared int the pair
// passes the row's last state through.
template <int K>
__device__ void sweep_row(const SweepParams &p, int row, double *tr, unsigned char *wv, int *st_slot, int pair) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int pt = (warp & 1) * 32 + lane, bar = 1 + pair;
    const bool lead = (warp & 1) == 0;  // the pair's first warp settles and refits the row
    u64 cv[PairTrellis<K>::NB][PairTrellis<K>::RT / 2];
    const double *tab = p.tables + (K - 1) * kStates;
    load_pair_values<K>(tab, pt, cv);
    float *best0 = reinterpret_cast<float *>(wv);
    float *best1 = best0 + PairTrellis<K>::R;
    uint32_t *args = reinterpret_cast<uint32_t *>(best1 + PairTrellis<K>::R);
    float *red = reinterpret_cast<float *>(wv + kPairMax);
    const int n = p.n, b0 = p.b0, b1 = p.b1;
    const double s = p.S[row];
    double *Trow = p.T + (int64_t)row * p.ldT;
    // every row's path starts at state 0 (codes.py:399-400), later runs where the last one ended
    int start = b0 > 0 ? p.rstate[row] : 0;
    if (p.dead != nullptr && b0 == 0)  // dead inputs: their targets start at zero (syntax.py:100-101)
        for (int c = pt; c < n; c += 64)
            if (p.dead[c]) Trow[c] = 0.0;
    const int ncol = b1 - b0 + min(p.look, n - b1);
    for (int c = pt; c < ncol; c += 64) tr[c] = Trow[b0 + c];  // the same thread zeroed its dead columns above
    pair_sync(bar);
    for (int j = b0; j < b1; j += p.width) {
        const int w = min(p.width, n - j);
        const int win = w + min(p.look, n - j - w);
        const double tv = (lane < win) ? tr[j - b0 + lane] : 0.0;
        const float xv = __double2float_rn(__ddiv_rn(tv, s));  // (T / S).to(float32)
        const int st = viterbi_window_pair<K>(xv, win, start, pt, bar, cv, best0, best1, args, red);
        if (lead) {
            const int last = __shfl_sync(0xffffffffu, st, w - 1);
            double e = 0.0;
            if (lane < w) {
                const double q = __ldg(tab + st);  // the fp64 table value (codes.py:404)
                p.states[(int64_t)row * n + j + lane] = (int16_t)st;
                if (p.settled != nullptr) p.settled[(int64_t)row * n + j + lane] = q;
                Trow[j + lane] = tv;                        // the column as it stood (sweep's return value)
                e = __dsub_rn(tv, __dmul_rn(q, s));         // E = T - q·S (codes.py:449, syntax.py:115)
            }
            // z·U_BB = E, U_BB upper triangular: column-by-column substitution (syntax.py:117). Lane c keeps column c
            // of U_BB in registers and the reciprocal of its diagonal, so the dependent chain is one multiply and one
            // fused update per column.
            double ucol[16];
#pragma unroll
            for (int i = 0; i < 16; ++i)
                ucol[i] = (i < w && lane < w) ? __ldg(p.U + (int64_t)(j + i) * p.ldU + j + lane) : 0.0;
            const double rdiag = (lane < w) ? 1.0 / __ldg(p.U + (int64_t)(j + lane) * p.ldU + j + lane) : 0.0;
            double acc = e;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                if (i < w) {
                    const double zi = __shfl_sync(0xffffffffu, acc * rdiag, i);
                    if (lane > i && lane < w) acc = fma(-zi, ucol[i], acc);
                    if (lane == i) acc = zi;
                }
            }
            __syncwarp();
            if (lane < w) tr[j - b0 + lane] = acc;  // the block's slots now hold z
            if (lane == 0) *st_slot = last;
        }
        pair_sync(bar);  // z and the new start state are visible to the pair
        start = *st_slot;
        // the rest of the run: T[j+w : b1] -= z · U[block, j+w : b1] (syntax.py:118), both warps of the pair
        for (int c = j + w + pt; c < b1; c += 64) {
            double a = 0.0;
            for (int i = 0; i < w; ++i) a = fma(tr[j - b0 + i], __ldg(p.U + (int64_t)(j + i) * p.ldU + c), a);
            tr[c - b0] -= a;
        }
        pair_sync(bar);  // the next window reads the updated run
    }
    // the run's z (the Trun slots of its columns) and the row's last state, for the run product and the next run
    for (int c = pt; c < b1 - b0; c += 64) p.Z[(int64_t)row * kMaxLazy + c] = tr[c];
    if (pt == 0) p.rstate[row] = start;
    pair_sync(bar);  // the slot is free for the pair's next row
}

__global__ void __launch_bounds__(kThreads, 1) sweep_run_kernel(SweepParams p) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int pair = warp >> 1, pt = (warp & 1) * 32 + lane, bar = 1 + pair;
    double *tr = reinterpret_cast<double *>(smem) + (size_t)pair * p.trun_stride;
    unsigned char *uni = smem + (size_t)kPairs * p.trun_stride * sizeof(double);
    uni = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(uni) + 15) & ~uintptr_t(15));
    unsigned char *wv = uni + (size_t)pair * kPairViterbiBytes;
    __shared__ int row_s[kPairs], st_s[kPairs];
    const int nrows = *p.nrows;
    const int spread = gridDim.x * kPairs;
    // first round: row pair·grid + CTA, so a short list lands on every SM before any SM takes a second row
    int idx = pair * gridDim.x + blockIdx.x;
    for (;;) {
        if (idx >= nrows) break;
        const int row = p.rowlist[idx];
        const int k = p.row_bits ? (int)p.row_bits[row] : p.k_all;
        switch (k) {
            case 1: sweep_row<1>(p, row, tr, wv, st_s + pair, pair); break;
            case 2: sweep_row<2>(p, row, tr, wv, st_s + pair, pair); break;
            case 3: sweep_row<3>(p, row, tr, wv, st_s + pair, pair); break;
            default: sweep_row<4>(p, row, tr, wv, st_s + pair, pair); break;
        }
        if (pt == 0) row_s[pair] = spread + atomicAdd(p.counters + p.run, 1);
        pair_sync(bar);
        idx = row_s[pair];
    }
}

// Lists rows grouped by width, the widest first (their rows take longest, so the persistent grid ends on the short
// ones), ascending row order inside each width (tile_rows = 1: no padding); one CTA.
__global__ void group_rows_kernel(int64_t rows, const uint8_t *row_bits, int k_all, int tile_rows, int32_t *rowlist,
                                  int *nlisted, int *counters, int nruns) {
    __shared__ int base[5];
    __shared__ int warp_sums[32];
    int cursor = 0;
    const int tid = threadIdx.x, nt = blockDim.x;
    for (int k = 4; k >= 1; --k) {
        // ascending scan of rows with width k
        int offset = 0;
        for (int64_t a = 0; a < rows; a += nt) {
            const int64_t r = a + tid;
            const int kr = r < rows ? (row_bits ? (int)row_bits[r] : k_all) : 0;
            const int flag = (kr == k) ? 1 : 0;
            // block-wide exclusive scan of flag
            const unsigned ballot = __ballot_sync(0xffffffffu, flag);
            const int lane = tid & 31, wid = tid >> 5;
            const int before_in_warp = __popc(ballot & ((1u << lane) - 1u));
            if (lane == 0) warp_sums[wid] = __popc(ballot);
            __syncthreads();
            int before_warps = 0, total = 0;
            for (int w = 0; w < nt / 32; ++w) {
                if (w < wid) before_warps += warp_sums[w];
                total += warp_sums[w];
            }
            if (flag) rowlist[cursor + offset + before_warps + before_in_warp] = (int32_t)r;
            offset += total;
            __syncthreads();
        }
        const int padded = (offset + tile_rows - 1) / tile_rows * tile_rows;
        for (int i = offset + tid; i < padded; i += nt) rowlist[cursor + i] = -1;
        cursor += padded;
        __syncthreads();
    }
    if (tid == 0) *nlisted = cursor / tile_rows;
    for (int r = tid; r < nruns; r += nt) counters[r] = 0;
    (void)base;
}

}  // namespace

}  // namespace lamq

using namespace lamq;

// Workspace: the tile list, per-run tile counters, each row's last state and the run's z per row.
struct SweepLayout {
    size_t rowlist, counters, rstate, z, total;
};

static SweepLayout sweep_layout(int64_t rows, int n) {
    auto up = [](size_t b) { return (b + 255) / 256 * 256; };
    SweepLayout l{};
    l.rowlist = up((size_t)(rows + 2) * sizeof(int32_t));  // + the row count
    l.counters = up((size_t)((n + 3) / 4 + 1) * sizeof(int));             // runs are at least 4 columns
    l.rstate = up((size_t)rows * sizeof(int));
    l.z = up((size_t)rows * kMaxLazy * sizeof(double));
    l.total = l.rowlist + l.counters + l.rstate + l.z;
    return l;
}

extern "C" size_t lamq_ldlq_rowtrellis_workspace_size(int64_t rows, int n) {
    if (rows <= 0 || n <= 0) return 0;
    return sweep_layout(rows, n).total;
}

extern "C" int lamq_ldlq_rowtrellis(double *T, int64_t ldT, int64_t rows, int n, const double *U, int64_t ldU,
                                    const uint8_t *dead, const double *S, const double *tables,
                                    const uint8_t *row_bits, int k_all, int L, int width, int look, int lazy,
                                    int16_t *states, double *settled, void *workspace, size_t workspace_bytes,
                                    lamq_stream_t stream) {
    LAMQ_REQUIRE(L == kL, "lamq_ldlq_rowtrellis: only L = 12 is supported (got %d)", L);
    LAMQ_REQUIRE(rows >= 0 && n >= 0, "lamq_ldlq_rowtrellis: negative shape");
    if (rows == 0 || n == 0) return LAMQ_OK;
    LAMQ_REQUIRE(T && U && S && tables && states, "lamq_ldlq_rowtrellis: null pointer");
    LAMQ_REQUIRE(ldT >= n && ldU >= n, "lamq_ldlq_rowtrellis: leading dimension below n");
    LAMQ_REQUIRE(width >= 1 && look >= 0 && width + look <= kMaxWin, "lamq_ldlq_rowtrellis: need width + look <= 24");
    LAMQ_REQUIRE(lazy >= width && lazy % width == 0 && lazy <= kMaxLazy && lazy % 4 == 0,
                 "lamq_ldlq_rowtrellis: lazy must be a multiple of width and of 4, at most 128");
    LAMQ_REQUIRE(row_bits != nullptr || (k_all >= 1 && k_all <= 4), "lamq_ldlq_rowtrellis: k must be 1..4");
    LAMQ_REQUIRE(rows <= INT32_MAX, "lamq_ldlq_rowtrellis: too many rows");
    const SweepLayout l = sweep_layout(rows, n);
    LAMQ_REQUIRE(workspace != nullptr && workspace_bytes >= l.total,
                 "lamq_ldlq_rowtrellis: workspace of %zu bytes needed, %zu given", l.total, workspace_bytes);
    cudaStream_t s = (cudaStream_t)stream;
    uint8_t *base = reinterpret_cast<uint8_t *>(workspace);
    int32_t *rowlist = reinterpret_cast<int32_t *>(base);
    int *nrows = reinterpret_cast<int *>(rowlist + rows);
    int *counters = reinterpret_cast<int *>(base + l.rowlist);
    int *rstate = reinterpret_cast<int *>(base + l.rowlist + l.counters);
    double *Z = reinterpret_cast<double *>(base + l.rowlist + l.counters + l.rstate);
    const int nruns = (n + lazy - 1) / lazy;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    group_rows_kernel<<<1, 1024, 0, s>>>(rows, row_bits, k_all, 1, rowlist, nrows, counters, nruns);
    LAMQ_CHECK_LAUNCH("lamq_ldlq_rowtrellis (grouping)");
    // Trun rows of lazy + look doubles, padded to an odd number of 16-byte units (conflict-free row starts)
    int ts = lazy + look;
    while ((2 * ts) % 32 != 24) ++ts;
    SweepParams p{T, ldT, n, rowlist, nrows, counters, row_bits, k_all, U, ldU, dead, S, tables,
                  width, look, lazy, ts, Z, rstate, 0, 0, 0, states, settled};
    const size_t smem = (size_t)kPairs * ts * sizeof(double) + 16 + kUnionBytes;
    cudaError_t e = smem_limit_max_once((const void *)sweep_run_kernel);
    if (e != cudaSuccess) {
        set_error("lamq_ldlq_rowtrellis: %s", cudaGetErrorString(e));
        return LAMQ_ERR_CUDA;
    }
    // one CTA per SM (fewer when there are fewer rows than SMs)
    const int grid = (int)std::min<int64_t>(sms, rows);
    for (int run = 0; run < nruns; ++run) {
        p.run = run;
        p.b0 = run * lazy;
        p.b1 = std::min(p.b0 + lazy, n);
        sweep_run_kernel<<<grid, kThreads, smem, s>>>(p);
        LAMQ_CHECK_LAUNCH("lamq_ldlq_rowtrellis");
        if (p.b1 < n) {  // the run's errors reach every later column: T[:, b1:] −= Z·U[b0:b1, b1:]
            const int st = lamq_dgemm(0, (int)rows, n - p.b1, p.b1 - p.b0, -1.0, Z, kMaxLazy,
                                      U + (int64_t)p.b0 * ldU + p.b1, ldU, 1.0, T + p.b1, ldT, stream);
            if (st != LAMQ_OK) return st;
        }
    }
    return LAMQ_OK;
}
