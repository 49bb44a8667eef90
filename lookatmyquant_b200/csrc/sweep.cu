// The block-LDLQ sweep with a row trellis (the lm2 build's per-matrix loop), fused into one kernel.
//
// Reference: opgraph/syntax.py:86-124 (`sweep`), with the projection of opgraph/codes.py:442-450 and
// RowTrellisCode.step (codes.py:397-404). Rows never interact under Refit (codes.py:417-418), so each row is settled
// start to finish by one warp with no synchronisation beyond the warp: for every block of `width` columns the warp
// decodes the block plus `look` columns ahead (in units of the row scale, from the row's previous state), settles the
// block, solves z·U_BB = E and carries the error into the rest of the run; after each run of `lazy` columns it
// carries the run's errors into all later columns. The look-ahead columns past a run's end are read before that
// end-of-run update, exactly as the reference reads them (stale by design).
#include <algorithm>

#include "lamq_common.cuh"
#include "trellis_warp.cuh"

namespace lamq {

namespace {

constexpr int kSweepWarps = 8;

struct SweepParams {
    double *T;
    int64_t ldT;
    int64_t rows;
    int n;
    const double *U;
    int64_t ldU;
    const uint8_t *dead;
    const double *S;
    const double *tables;
    const uint8_t *row_bits;
    int k_all;
    int width, look, lazy;
    int16_t *states;
    double *settled;
};

__host__ __device__ constexpr size_t sweep_warp_smem(int win, int lazy) {
    return 2 * 2048 * sizeof(float) + (size_t)win * 32 * sizeof(unsigned long long) + (size_t)lazy * sizeof(double);
}

template <int K>
__device__ void sweep_row(const SweepParams &p, int64_t row, int lane, float *best0, float *best1,
                          unsigned long long *args, double *Z) {
    float cv[Trellis<K>::NB][Trellis<K>::RL];
    const double *tab = p.tables + (K - 1) * kStates;
    load_pred_values<K>(tab, lane, cv);
    const int n = p.n;
    double *Trow = p.T + row * p.ldT;
    const double s = p.S[row];
    const double *U = p.U;
    const int64_t ldU = p.ldU;
    if (p.dead != nullptr)
        for (int c = lane; c < n; c += 32)
            if (p.dead[c]) Trow[c] = 0.0;
    __syncwarp();
    int state = 0;  // RowTrellisCode.step: every row's path starts at state 0 (codes.py:399-400)
    for (int b0 = 0; b0 < n; b0 += p.lazy) {
        const int b1 = min(b0 + p.lazy, n);
        for (int j = b0; j < b1; j += p.width) {
            const int w = min(p.width, n - j);
            const int win = w + min(p.look, n - j - w);
            const double tv = (lane < win) ? Trow[j + lane] : 0.0;
            const float xv = __double2float_rn(__ddiv_rn(tv, s));  // (T / S).to(float32)
            const int st = viterbi_window<K>(xv, win, true, state, cv, best0, best1, args, lane);
            state = __shfl_sync(0xffffffffu, st, w - 1);
            double e = 0.0;
            if (lane < w) {
                const double q = __ldg(tab + st);  // the fp64 table value (codes.py:404)
                p.states[row * (int64_t)n + j + lane] = (int16_t)st;
                if (p.settled != nullptr) p.settled[row * (int64_t)n + j + lane] = q;
                e = __dsub_rn(tv, __dmul_rn(q, s));  // E = T - q·S (codes.py:449, syntax.py:115)
            }
            // z·U_BB = E, U_BB upper triangular: column-by-column substitution (syntax.py:117)
            double acc = e;
            for (int i = 0; i < w; ++i) {
                const double zi = __ddiv_rn(__shfl_sync(0xffffffffu, acc, i), U[(int64_t)(j + i) * ldU + j + i]);
                if (lane == i) Z[j - b0 + i] = zi;
                if (lane > i && lane < w) acc = __dsub_rn(acc, __dmul_rn(zi, U[(int64_t)(j + i) * ldU + j + lane]));
            }
            __syncwarp();
            // the rest of the run: T[j+w : b1] -= z · U[block, j+w : b1] (syntax.py:118)
            for (int c = j + w + lane; c < b1; c += 32) {
                double a = 0.0;
                for (int i = 0; i < w; ++i) a = fma(Z[j - b0 + i], U[(int64_t)(j + i) * ldU + c], a);
                Trow[c] -= a;
            }
            __syncwarp();
        }
        if (b1 < n) {  // the columns after the run: T[b1:] -= Z · U[b0:b1, b1:] (syntax.py:122-123)
            const int nr = b1 - b0;
            for (int c = b1 + lane; c < n; c += 32) {
                double a = 0.0;
                for (int i = 0; i < nr; ++i) a = fma(Z[i], U[(int64_t)(b0 + i) * ldU + c], a);
                Trow[c] -= a;
            }
            __syncwarp();
        }
    }
}

__global__ void __launch_bounds__(kSweepWarps * 32, 1) sweep_rowtrellis_kernel(SweepParams p) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * kSweepWarps + warp;
    if (row >= p.rows) return;
    const int win = p.width + p.look;
    unsigned char *base = smem + (size_t)warp * sweep_warp_smem(win, p.lazy);
    float *best0 = reinterpret_cast<float *>(base);
    float *best1 = best0 + 2048;
    unsigned long long *args = reinterpret_cast<unsigned long long *>(best1 + 2048);
    double *Z = reinterpret_cast<double *>(args + win * 32);
    const int k = p.row_bits != nullptr ? (int)p.row_bits[row] : p.k_all;
    switch (k) {
        case 1: sweep_row<1>(p, row, lane, best0, best1, args, Z); break;
        case 2: sweep_row<2>(p, row, lane, best0, best1, args, Z); break;
        case 3: sweep_row<3>(p, row, lane, best0, best1, args, Z); break;
        case 4: sweep_row<4>(p, row, lane, best0, best1, args, Z); break;
        default:  // an invalid width: mark the row's states invalid rather than guess
            for (int c = lane; c < p.n; c += 32) p.states[row * (int64_t)p.n + c] = -1;
    }
}

}  // namespace

}  // namespace lamq

using namespace lamq;

extern "C" int lamq_ldlq_rowtrellis(double *T, int64_t ldT, int64_t rows, int n, const double *U, int64_t ldU,
                                    const uint8_t *dead, const double *S, const double *tables,
                                    const uint8_t *row_bits, int k_all, int L, int width, int look, int lazy,
                                    int16_t *states, double *settled, lamq_stream_t stream) {
    LAMQ_REQUIRE(L == kL, "lamq_ldlq_rowtrellis: only L = 12 is supported (got %d)", L);
    LAMQ_REQUIRE(rows >= 0 && n >= 0, "lamq_ldlq_rowtrellis: negative shape");
    if (rows == 0 || n == 0) return LAMQ_OK;
    LAMQ_REQUIRE(T && U && S && tables && states, "lamq_ldlq_rowtrellis: null pointer");
    LAMQ_REQUIRE(ldT >= n && ldU >= n, "lamq_ldlq_rowtrellis: leading dimension below n");
    LAMQ_REQUIRE(width >= 1 && look >= 0 && width + look <= 32, "lamq_ldlq_rowtrellis: need width + look <= 32");
    LAMQ_REQUIRE(lazy >= width && lazy % width == 0 && lazy <= 256,
                 "lamq_ldlq_rowtrellis: lazy must be a multiple of width, at most 256");
    LAMQ_REQUIRE(row_bits != nullptr || (k_all >= 1 && k_all <= 4), "lamq_ldlq_rowtrellis: k must be 1..4");
    SweepParams p{T, ldT, rows, n, U, ldU, dead, S, tables, row_bits, k_all, width, look, lazy, states, settled};
    const size_t smem = kSweepWarps * sweep_warp_smem(width + look, lazy);
    cudaError_t e = cudaFuncSetAttribute(sweep_rowtrellis_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) {
        set_error("lamq_ldlq_rowtrellis: %s", cudaGetErrorString(e));
        return LAMQ_ERR_CUDA;
    }
    const int64_t grid = (rows + kSweepWarps - 1) / kSweepWarps;
    sweep_rowtrellis_kernel<<<(unsigned)grid, kSweepWarps * 32, smem, (cudaStream_t)stream>>>(p);
    LAMQ_CHECK_LAUNCH("lamq_ldlq_rowtrellis");
    return LAMQ_OK;
}
