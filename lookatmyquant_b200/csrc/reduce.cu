// Sums of squares over the rows or the columns of an activation or gradient matrix, in fp64: the per-output-channel
// E[y²] and E[g²] of row importance (row_importance.py:57-93: yy += Σ_tokens y², gg += Σ_tokens g²) and the
// per-token Σ_channels g² of GuidedQuant's token weights (quantize.py:853-894).
//
// Column sums: chunks of kChunkRows rows are summed by separate blocks (a thread per column, coalesced reads) into
// fp64 partials, which a second kernel adds chunk by chunk in order into the accumulator: the result does not depend
// on the launch shape and repeated calls agree bit for bit. Row sums: a warp per row, lanes strided over the columns,
// a fixed shuffle tree.
#include <algorithm>
#include <cstdint>

#include <cuda_bf16.h>

#include "lamq_common.cuh"

namespace lamq {
namespace {

constexpr int kChunkRows = 256;
constexpr int kColThreads = 256;

template <typename T>
__device__ __forceinline__ double sq(const T *p) {
    const double v = (double)static_cast<float>(*p);
    return v * v;
}

template <>
__device__ __forceinline__ double sq<__nv_bfloat16>(const __nv_bfloat16 *p) {
    const double v = (double)__bfloat162float(*p);
    return v * v;
}

template <typename T>
__global__ void col_partials_kernel(const T *__restrict__ x, int64_t rows, int cols, int64_t ld,
                                    double *__restrict__ part) {
    const int j = blockIdx.x * kColThreads + threadIdx.x;
    const int64_t chunk = blockIdx.y;
    if (j >= cols) return;
    const int64_t r0 = chunk * kChunkRows, r1 = std::min<int64_t>(rows, r0 + kChunkRows);
    double acc = 0.0;
    for (int64_t r = r0; r < r1; ++r) acc += sq(x + r * ld + j);
    part[chunk * cols + j] = acc;
}

__global__ void col_total_kernel(const double *__restrict__ part, int64_t chunks, int cols, double *__restrict__ out) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= cols) return;
    double acc = 0.0;
    for (int64_t c = 0; c < chunks; ++c) acc += part[c * cols + j];
    out[j] += acc;
}

template <typename T>
__global__ void row_sums_kernel(const T *__restrict__ x, int64_t rows, int cols, int64_t ld, double *__restrict__ out) {
    const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const T *p = x + row * ld;
    double acc = 0.0;
    for (int j = lane; j < cols; j += 32) acc += sq(p + j);
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_down_sync(0xffffffffu, acc, o);
    if (lane == 0) out[row] = acc;
}

template <typename T>
int run(const void *xv, int64_t rows, int cols, int64_t ld, double *col_acc, double *row_out, void *ws,
        cudaStream_t s) {
    const T *x = reinterpret_cast<const T *>(xv);
    if (col_acc) {
        const int64_t chunks = (rows + kChunkRows - 1) / kChunkRows;
        LAMQ_REQUIRE(chunks <= 65535, "lamq_square_sums: %lld rows exceed %d chunks of %d", (long long)rows, 65535,
                     kChunkRows);
        double *part = reinterpret_cast<double *>(ws);
        dim3 grid((cols + kColThreads - 1) / kColThreads, (unsigned)chunks);
        col_partials_kernel<T><<<grid, kColThreads, 0, s>>>(x, rows, cols, ld, part);
        LAMQ_CHECK_LAUNCH("lamq_square_sums columns");
        col_total_kernel<<<(cols + 255) / 256, 256, 0, s>>>(part, chunks, cols, col_acc);
        LAMQ_CHECK_LAUNCH("lamq_square_sums columns total");
    }
    if (row_out) {
        const int64_t blocks = (rows * 32 + 255) / 256;
        LAMQ_REQUIRE(blocks <= INT32_MAX, "lamq_square_sums: too many rows");
        row_sums_kernel<T><<<(unsigned)blocks, 256, 0, s>>>(x, rows, cols, ld, row_out);
        LAMQ_CHECK_LAUNCH("lamq_square_sums rows");
    }
    return LAMQ_OK;
}

}  // namespace
}  // namespace lamq

using namespace lamq;

extern "C" size_t lamq_square_sums_workspace_size(int64_t rows, int cols) {
    if (rows <= 0 || cols <= 0) return 0;
    return (size_t)((rows + kChunkRows - 1) / kChunkRows) * (size_t)cols * sizeof(double);
}

extern "C" int lamq_square_sums(const void *x, int dtype, int64_t rows, int cols, int64_t ld, double *col_acc,
                                double *row_out, void *workspace, size_t workspace_bytes, lamq_stream_t stream) {
    LAMQ_REQUIRE(rows >= 0 && cols >= 0 && ld >= cols, "lamq_square_sums: bad shape");
    LAMQ_REQUIRE(dtype == LAMQ_F32 || dtype == LAMQ_BF16, "lamq_square_sums: dtype must be LAMQ_F32 or LAMQ_BF16");
    if (rows == 0 || cols == 0) return LAMQ_OK;
    LAMQ_REQUIRE(x && (col_acc || row_out), "lamq_square_sums: null pointer");
    LAMQ_REQUIRE(!col_acc || (workspace && workspace_bytes >= lamq_square_sums_workspace_size(rows, cols)),
                 "lamq_square_sums: workspace of %zu bytes needed", lamq_square_sums_workspace_size(rows, cols));
    cudaStream_t s = (cudaStream_t)stream;
    return dtype == LAMQ_F32 ? run<float>(x, rows, cols, ld, col_acc, row_out, workspace, s)
                             : run<__nv_bfloat16>(x, rows, cols, ld, col_acc, row_out, workspace, s);
}
