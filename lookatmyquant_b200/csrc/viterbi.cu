// Standalone Viterbi over the 12-bit bitshift trellis: opgraph/codes.py:151-181 (`viterbi`), one warp per row.
//
// Used for whole-row decodes (RowTrellisCode.apply without a sweep, codes.py:406-410), the column runs of
// TrellisCode.project (codes.py:375-378) and the kernel-level parity tests. Sequences of up to 32 entries keep their
// back-pointers in shared memory; longer ones keep them in the caller's workspace (256 bytes per entry per row).
#include "lamq_common.cuh"
#include "trellis_warp.cuh"

namespace lamq {

namespace {

constexpr int kVitWarps = 8;
constexpr int kShortT = 32;

struct VitParams {
    const float *X;
    int64_t rows;
    int T;
    const float *values;
    const int64_t *start;
    int64_t *states;
    unsigned long long *gargs;  // rows x T x 32 back-pointer words, or null when T <= kShortT
};

template <int K>
__device__ void viterbi_row(const VitParams &p, int64_t row, int lane, float *best0, float *best1,
                            unsigned long long *args) {
    float cv[Trellis<K>::NB][Trellis<K>::RL];
    load_pred_values_f32<K>(p.values, lane, cv);
    const float *x = p.X + row * (int64_t)p.T;
    const int T = p.T;
    const bool has_start = p.start != nullptr;
    const int start = has_start ? (int)(p.start[row] & (kStates - 1)) : 0;
    init_best<K>(best0, lane, has_start, start);
    __syncwarp();
    float *bin = best0, *bout = best1;
    for (int t = 1; t < T; ++t) {
        const float xp = __ldg(x + t - 1);
        args[(int64_t)t * 32 + lane] = acs_step<K>(bin, bout, xp, lane, cv);
        __syncwarp();
        float *tmp = bin;
        bin = bout;
        bout = tmp;
    }
    const int fs = final_argmin<K>(bin, __ldg(x + T - 1), lane, cv);
    __syncwarp();
    int64_t *out = p.states + row * (int64_t)T;
    using Tr = Trellis<K>;
    int s = fs;
    if (lane == 0) out[T - 1] = s;
    for (int t = T - 1; t > 0; --t) {
        const int r = s >> K;
        const unsigned long long w = args[(int64_t)t * 32 + r / Tr::RL];
        s = (int)((w >> ((r % Tr::RL) * K)) & (Tr::NB - 1)) * Tr::R + r;
        if (lane == 0) out[t - 1] = s;
    }
}

__global__ void __launch_bounds__(kVitWarps * 32, 1) viterbi_kernel(VitParams p, int k) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * kVitWarps + warp;
    if (row >= p.rows) return;
    const size_t per_warp = 2 * 2048 * sizeof(float) + (p.gargs ? 0 : (size_t)kShortT * 32 * 8);
    unsigned char *base = smem + warp * per_warp;
    float *best0 = reinterpret_cast<float *>(base);
    float *best1 = best0 + 2048;
    unsigned long long *args = p.gargs ? p.gargs + row * (int64_t)p.T * 32
                                       : reinterpret_cast<unsigned long long *>(best1 + 2048);
    switch (k) {
        case 1: viterbi_row<1>(p, row, lane, best0, best1, args); break;
        case 2: viterbi_row<2>(p, row, lane, best0, best1, args); break;
        case 3: viterbi_row<3>(p, row, lane, best0, best1, args); break;
        default: viterbi_row<4>(p, row, lane, best0, best1, args); break;
    }
}

}  // namespace

}  // namespace lamq

using namespace lamq;

extern "C" size_t lamq_viterbi_workspace_size(int64_t rows, int T, int L, int k) {
    (void)L;
    (void)k;
    if (rows <= 0 || T <= kShortT) return 0;
    return (size_t)rows * (size_t)T * 32 * sizeof(unsigned long long);
}

extern "C" int lamq_viterbi(const float *X, int64_t rows, int T, const float *values, int L, int k,
                            const int64_t *start, int64_t *states, void *workspace, size_t workspace_bytes,
                            lamq_stream_t stream) {
    LAMQ_REQUIRE(L == kL, "lamq_viterbi: only L = 12 is supported (got %d)", L);
    LAMQ_REQUIRE(k >= 1 && k <= 4, "lamq_viterbi: k must be 1..4 (got %d)", k);
    LAMQ_REQUIRE(rows >= 0 && T >= 0, "lamq_viterbi: negative shape");
    if (rows == 0 || T == 0) return LAMQ_OK;
    LAMQ_REQUIRE(X && values && states, "lamq_viterbi: null pointer");
    const size_t need = lamq_viterbi_workspace_size(rows, T, L, k);
    LAMQ_REQUIRE(workspace_bytes >= need && (need == 0 || workspace != nullptr),
                 "lamq_viterbi: workspace of %zu bytes needed, %zu given", need, workspace_bytes);
    VitParams p{X, rows, T, values, start, states,
                need ? reinterpret_cast<unsigned long long *>(workspace) : nullptr};
    const size_t per_warp = 2 * 2048 * sizeof(float) + (need ? 0 : (size_t)kShortT * 32 * 8);
    const size_t smem = kVitWarps * per_warp;
    cudaError_t e = cudaFuncSetAttribute(viterbi_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) {
        set_error("lamq_viterbi: %s", cudaGetErrorString(e));
        return LAMQ_ERR_CUDA;
    }
    const int64_t grid = (rows + kVitWarps - 1) / kVitWarps;
    viterbi_kernel<<<(unsigned)grid, kVitWarps * 32, smem, (cudaStream_t)stream>>>(p, k);
    LAMQ_CHECK_LAUNCH("lamq_viterbi");
    return LAMQ_OK;
}
