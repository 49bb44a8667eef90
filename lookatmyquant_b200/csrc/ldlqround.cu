// Scalar-level LDLQ rounding (GPTQ's lazy-batch form) in fp64: the GPU rounding of the reference's nested.py path.
//
// Reference: opgraph/ldlq_gpu.py:29-49 (`ldlq_round`): inside a block of `block` inputs every row takes its inputs in
// order — q = levels[bucketize(x, mids)] (mids the midpoints of the sorted levels), e = (x − q) / U[j][j], the block's
// later inputs x_c −= e·U[j][c] — and the block's errors reach the inputs after it through one product,
// X[:, b:] −= Err·U[a:b, b:].
//
// Rows never interact inside a block, so one thread takes one row: round_block_kernel stages the block's U (upper
// triangle) and the CTA's rows of the block (transposed, so consecutive threads read consecutive words) in shared
// memory and walks the block's columns with the reference's separately rounded fp64 operations; the product after the
// block is lamq_dgemm.
#include <algorithm>

#include "lamq_common.cuh"

namespace lamq {
namespace {

constexpr int kRoundRows = 64;    // rows (threads) per CTA
constexpr int kRoundBlock = 128;  // largest block
constexpr int kRoundLevels = 1024;
constexpr int kXsLd = kRoundRows + 1;  // the staged rows' stride (doubles): column-wise writes spread over the banks

__global__ void __launch_bounds__(kRoundRows) round_block_kernel(const double *__restrict__ X, int64_t ldX,
                                                                int64_t rows, const double *__restrict__ U,
                                                                int64_t ldU, int a, int bw,
                                                                const double *__restrict__ levels, int nl,
                                                                double *__restrict__ Q, int64_t ldQ,
                                                                double *__restrict__ Err) {
    extern __shared__ __align__(16) double rsm[];
    double *Ub = rsm;                       // bw x bw (upper part used)
    double *Xs = Ub + bw * bw;              // bw x kXsLd: Xs[c][r]
    double *lv = Xs + bw * kXsLd;           // nl levels
    double *mids = lv + nl;                 // nl − 1 midpoints
    const int t = threadIdx.x;
    for (int e = t; e < bw * bw; e += kRoundRows) {
        const int i = e / bw, c = e - i * bw;
        Ub[e] = (c >= i) ? U[(int64_t)(a + i) * ldU + a + c] : 0.0;
    }
    for (int i = t; i < nl; i += kRoundRows) lv[i] = levels[i];
    __syncthreads();
    for (int i = t; i + 1 < nl; i += kRoundRows) mids[i] = (lv[i + 1] + lv[i]) / 2;  // (levels[1:] + levels[:-1]) / 2
    const int64_t r0 = (int64_t)blockIdx.x * kRoundRows;
    for (int e = t; e < bw * kRoundRows; e += kRoundRows) {  // consecutive threads read consecutive columns
        const int r = e / bw, c = e - r * bw;
        Xs[c * kXsLd + r] = (r0 + r < rows) ? X[(r0 + r) * ldX + a + c] : 0.0;
    }
    __syncthreads();
    const int64_t row = r0 + t;
    if (row >= rows) return;
    for (int j = 0; j < bw; ++j) {
        const double x = Xs[j * kXsLd + t];
        // bucketize(x, mids): the number of midpoints strictly below x
        int lo = 0, hi = nl - 1;
        while (lo < hi) {
            const int mid = (lo + hi) >> 1;
            if (mids[mid] < x) lo = mid + 1;
            else hi = mid;
        }
        const double q = lv[lo];
        Q[row * ldQ + a + j] = q;
        const double e = __ddiv_rn(__dsub_rn(x, q), Ub[j * bw + j]);
        Err[row * kRoundBlock + j] = e;
        for (int c = j + 1; c < bw; ++c)
            Xs[c * kXsLd + t] = __dsub_rn(Xs[c * kXsLd + t], __dmul_rn(e, Ub[j * bw + c]));
    }
}

}  // namespace
}  // namespace lamq

using namespace lamq;

extern "C" size_t lamq_ldlq_round_workspace_size(int64_t rows) {
    return rows <= 0 ? 0 : (size_t)rows * kRoundBlock * sizeof(double);
}

extern "C" int lamq_ldlq_round(double *X, int64_t ldX, int64_t rows, int n, const double *U, int64_t ldU,
                               const double *levels, int nlevels, int block, double *Q, int64_t ldQ, void *workspace,
                               size_t workspace_bytes, lamq_stream_t stream) {
    LAMQ_REQUIRE(rows >= 0 && n >= 0 && ldX >= n && ldU >= n && ldQ >= n, "lamq_ldlq_round: bad shape");
    if (rows == 0 || n == 0) return LAMQ_OK;
    LAMQ_REQUIRE(nlevels >= 1 && nlevels <= kRoundLevels, "lamq_ldlq_round: 1..%d levels", kRoundLevels);
    LAMQ_REQUIRE(block >= 1 && block <= kRoundBlock, "lamq_ldlq_round: block in 1..%d", kRoundBlock);
    LAMQ_REQUIRE(X && U && levels && Q && workspace, "lamq_ldlq_round: null pointer");
    LAMQ_REQUIRE(workspace_bytes >= lamq_ldlq_round_workspace_size(rows), "lamq_ldlq_round: workspace too small");
    cudaStream_t s = (cudaStream_t)stream;
    double *Err = reinterpret_cast<double *>(workspace);
    const size_t smem = ((size_t)block * block + (size_t)block * kXsLd + 2 * (size_t)nlevels) * sizeof(double);
    const cudaError_t e = smem_limit_once((const void *)round_block_kernel,
                                          (int)(((size_t)kRoundBlock * kRoundBlock + (size_t)kRoundBlock * kXsLd +
                                                 2 * (size_t)kRoundLevels) * sizeof(double)));
    if (e != cudaSuccess) {
        set_error("lamq_ldlq_round: %s", cudaGetErrorString(e));
        return LAMQ_ERR_CUDA;
    }
    const unsigned grid = (unsigned)((rows + kRoundRows - 1) / kRoundRows);
    for (int a = 0; a < n; a += block) {
        const int b = std::min(a + block, n);
        round_block_kernel<<<grid, kRoundRows, smem, s>>>(X, ldX, rows, U, ldU, a, b - a, levels, nlevels, Q, ldQ,
                                                          Err);
        LAMQ_CHECK_LAUNCH("lamq_ldlq_round");
        if (b < n) {  // X[:, b:] −= Err · U[a:b, b:]
            const int rc = lamq_dgemm(0, (int)rows, n - b, b - a, -1.0, Err, kRoundBlock, U + (int64_t)a * ldU + b,
                                      ldU, 1.0, X + b, ldX, stream);
            if (rc != LAMQ_OK) return rc;
        }
    }
    return LAMQ_OK;
}
