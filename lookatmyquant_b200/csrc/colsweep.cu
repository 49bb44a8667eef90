// Column-trellis LDLQ sweep: the `sweep` of opgraph/syntax.py:86-124 with TrellisCode.project (opgraph/codes.py:
// 363-383) as the projection — the `measure` path's trellis words.
//
// Per block of `width` columns (inside runs of `lazy` columns):
//   1. each column of the block is cut into runs of Tm consecutive rows, and every run (an fp32 sequence of
//      T/S values) goes onto its nearest free-start trellis path — the lamq_viterbi kernel over all runs at once;
//   2. the refit, one warp per row: E = T[:, block] − V[states]·S, z·U_BB = E by substitution, the rest of the run
//      T[:, j+w : b1] −= z·U[block, j+w : b1], z kept for the end of the run;
//   3. at the end of a run, T[:, b1:] −= Z·U[b0:b1, b1:] (lamq_dgemm on the fp64 tensor cores).
// Rows couple only inside a run of Tm rows of one column (the Viterbi), so unlike the row sweep the blocks are global
// steps: the host walks the blocks and each step is a few launches over every row.
#include <algorithm>

#include "lamq_common.cuh"

namespace lamq {
namespace {

constexpr int kColMaxWidth = 32;  // a block's columns sit in one warp's lanes

// Working copy of T with dead inputs zeroed (syntax.py:100-101), and the fp32 table for the Viterbi.
__global__ void col_prep_kernel(const double *__restrict__ T, int64_t ldT, int64_t rows, int n,
                                const uint8_t *__restrict__ dead, double *__restrict__ Wk, const double *__restrict__ table,
                                int nt, float *__restrict__ table32) {
    const int64_t total = rows * n;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = e / n;
        const int c = (int)(e % n);
        Wk[e] = (dead != nullptr && dead[c]) ? 0.0 : T[r * ldT + c];
    }
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < nt; e += (int64_t)gridDim.x * blockDim.x)
        table32[e] = (float)table[e];
}

// Block columns [j, j + w): the "before" values out, and the Viterbi sequences: sequence (r / Tm)·w + c holds rows
// r of column j + c in order (codes.py:368-369), as fp32 T/S.
__global__ void col_gather_kernel(const double *__restrict__ Wk, int64_t rows, int n, int j, int w, int Tm,
                                  const double *__restrict__ S, double *__restrict__ before, int64_t ldT,
                                  float *__restrict__ xs) {
    const int64_t total = rows * w;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = e / w;
        const int c = (int)(e % w);
        const double v = Wk[r * n + j + c];
        before[r * ldT + j + c] = v;
        xs[((r / Tm) * w + c) * (int64_t)Tm + r % Tm] = __double2float_rn(__ddiv_rn(v, S[r]));
    }
}

// The refit of block [j, j + w) inside the run [b0, b1), one warp per row.
__global__ void col_refit_kernel(double *__restrict__ Wk, int64_t rows, int n, int j, int w, int b0, int b1, int Tm,
                                 const int64_t *__restrict__ st64, const double *__restrict__ table,
                                 const double *__restrict__ S, const double *__restrict__ U, int64_t ldU,
                                 int16_t *__restrict__ states, double *__restrict__ settled, double *__restrict__ Z,
                                 int ldz) {
    const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
    for (int64_t r = (int64_t)blockIdx.x * warps + (threadIdx.x >> 5); r < rows; r += (int64_t)gridDim.x * warps) {
        double *row = Wk + r * n;
        const double s = S[r];
        double e = 0.0;
        if (lane < w) {
            const int64_t st = st64[((r / Tm) * w + lane) * (int64_t)Tm + r % Tm];
            const double q = __ldg(table + st);
            states[r * n + j + lane] = (int16_t)st;
            if (settled != nullptr) settled[r * n + j + lane] = q;
            e = __dsub_rn(row[j + lane], __dmul_rn(q, s));  // E = T − q·S
        }
        // z·U_BB = E: column-by-column substitution, lane c keeping column c of U_BB
        const double rdiag = (lane < w) ? 1.0 / __ldg(U + (int64_t)(j + lane) * ldU + j + lane) : 0.0;
        double acc = e;
        for (int i = 0; i < w; ++i) {
            const double zi = __shfl_sync(0xffffffffu, acc * rdiag, i);
            if (lane > i && lane < w) acc = fma(-zi, __ldg(U + (int64_t)(j + i) * ldU + j + lane), acc);
            if (lane == i) acc = zi;
        }
        if (lane < w) Z[r * ldz + (j - b0) + lane] = acc;
        // the rest of the run: T[j+w : b1] −= z·U[block, j+w : b1]
        for (int c0 = j + w; c0 < b1; c0 += 32) {
            const int c = c0 + lane;
            double a = 0.0;
            for (int i = 0; i < w; ++i) {
                const double zi = __shfl_sync(0xffffffffu, acc, i);
                if (c < b1) a = fma(zi, __ldg(U + (int64_t)(j + i) * ldU + c), a);
            }
            if (c < b1) row[c] -= a;
        }
    }
}

int grid_for(int64_t work, int threads) { return (int)std::min<int64_t>((work + threads - 1) / threads, 148 * 16); }

struct ColLayout {
    size_t wk, xs, st, z, t32, vws, total;
};

ColLayout col_layout(int64_t rows, int n, int Tm, int L, int k, int width, int lazy) {
    auto up = [](size_t b) { return (b + 255) / 256 * 256; };
    ColLayout l{};
    const int64_t nseq = rows / Tm * width;
    l.wk = up((size_t)rows * n * sizeof(double));
    l.xs = up((size_t)rows * width * sizeof(float));
    l.st = up((size_t)rows * width * sizeof(int64_t));
    l.z = up((size_t)rows * lazy * sizeof(double));
    l.t32 = up(sizeof(float) << L);
    l.vws = up(lamq_viterbi_workspace_size(nseq, Tm, L, k));
    l.total = l.wk + l.xs + l.st + l.z + l.t32 + l.vws;
    return l;
}

}  // namespace
}  // namespace lamq

using namespace lamq;

extern "C" size_t lamq_ldlq_coltrellis_workspace_size(int64_t rows, int n, int Tm, int L, int k, int width, int lazy) {
    if (rows <= 0 || n <= 0 || Tm <= 0 || width <= 0 || lazy <= 0) return 0;
    return col_layout(rows, n, Tm, L, k, width, lazy).total;
}

extern "C" int lamq_ldlq_coltrellis(double *T, int64_t ldT, int64_t rows, int n, const double *U, int64_t ldU,
                                   const uint8_t *dead, const double *S, const double *table, int k, int L, int Tm,
                                   int width, int lazy, int16_t *states, double *settled, void *workspace,
                                   size_t workspace_bytes, lamq_stream_t stream) {
    LAMQ_REQUIRE(rows > 0 && n > 0 && ldT >= n && ldU >= n, "lamq_ldlq_coltrellis: bad shape");
    LAMQ_REQUIRE(Tm > 0 && rows % Tm == 0, "lamq_ldlq_coltrellis: rows (%lld) must be a multiple of the run length %d",
                 (long long)rows, Tm);
    LAMQ_REQUIRE(L == 12 && k >= 1 && k <= 4, "lamq_ldlq_coltrellis: supported L = 12, k in 1..4");
    LAMQ_REQUIRE(width >= 1 && width <= kColMaxWidth && lazy >= width && lazy % width == 0,
                 "lamq_ldlq_coltrellis: width in 1..32 and lazy a multiple of width");
    LAMQ_REQUIRE(T && U && S && table && states && workspace, "lamq_ldlq_coltrellis: null pointer");
    const ColLayout l = col_layout(rows, n, Tm, L, k, width, lazy);
    LAMQ_REQUIRE(workspace_bytes >= l.total, "lamq_ldlq_coltrellis: workspace too small");
    cudaStream_t s = (cudaStream_t)stream;
    uint8_t *base = reinterpret_cast<uint8_t *>(workspace);
    double *Wk = reinterpret_cast<double *>(base);
    float *xs = reinterpret_cast<float *>(base + l.wk);
    int64_t *st = reinterpret_cast<int64_t *>(base + l.wk + l.xs);
    double *Z = reinterpret_cast<double *>(base + l.wk + l.xs + l.st);
    float *t32 = reinterpret_cast<float *>(base + l.wk + l.xs + l.st + l.z);
    void *vws = base + l.wk + l.xs + l.st + l.z + l.t32;
    col_prep_kernel<<<grid_for(rows * n, 256), 256, 0, s>>>(T, ldT, rows, n, dead, Wk, table, 1 << L, t32);
    LAMQ_CHECK_LAUNCH("lamq_ldlq_coltrellis prep");
    for (int b0 = 0; b0 < n; b0 += lazy) {
        const int b1 = std::min(b0 + lazy, n);
        for (int j = b0; j < b1; j += width) {
            const int w = std::min(width, n - j);
            col_gather_kernel<<<grid_for(rows * w, 256), 256, 0, s>>>(Wk, rows, n, j, w, Tm, S, T, ldT, xs);
            LAMQ_CHECK_LAUNCH("lamq_ldlq_coltrellis gather");
            const int64_t nseq = rows / Tm * w;
            int rc = lamq_viterbi(xs, nseq, Tm, t32, L, k, nullptr, st, vws, l.vws, stream);
            if (rc != LAMQ_OK) return rc;
            col_refit_kernel<<<grid_for(rows * 32, 256), 256, 0, s>>>(Wk, rows, n, j, w, b0, b1, Tm, st, table, S, U,
                                                                      ldU, states, settled, Z, lazy);
            LAMQ_CHECK_LAUNCH("lamq_ldlq_coltrellis refit");
        }
        if (b1 < n) {
            const int rc = lamq_dgemm(0, (int)rows, n - b1, b1 - b0, -1.0, Z, lazy, U + (int64_t)b0 * ldU + b1, ldU, 1.0,
                                      Wk + b1, n, stream);
            if (rc != LAMQ_OK) return rc;
        }
    }
    return LAMQ_OK;
}
