// Standalone Viterbi over the 12-bit bitshift trellis: opgraph/codes.py:151-181 (`viterbi`), a warp (or a warp pair)
// per row.
//
// Used for whole-row decodes (RowTrellisCode.apply without a sweep, codes.py:406-410), the column runs of
// TrellisCode.project (codes.py:375-378) and the kernel-level parity tests. Sequences of up to 32 entries keep their
// back-pointers in shared memory; longer ones (the column runs: 256 or 320 entries, and only tens to hundreds of
// them per block) are decoded by a warp pair each (trellis_pair.cuh: half the states per thread, one back-pointer
// word per thread per step, all of them in shared memory), two sequences per CTA, unless their back-pointers do not
// fit; then one warp per sequence keeps them in the caller's workspace (256 bytes per entry per row).
#include <climits>
#include <cstdint>
#include <mutex>

#include "lamq_common.cuh"
#include "trellis_pair.cuh"
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

// A long sequence decoded by a warp pair (64 threads, pt = the thread's index in the pair): x, the two best buffers,
// every step's back-pointer words and the final reduction's scratch live in the pair's share of shared memory.
template <int K>
__device__ void viterbi_pair_long(const VitParams &p, int64_t row, int pair, int pt, unsigned char *base) {
    using Tr = PairTrellis<K>;
    const int T = p.T;
    float *xs = reinterpret_cast<float *>(base);
    float *best0 = xs + (T + 3) / 4 * 4;
    float *best1 = best0 + Tr::R;
    uint32_t *args = reinterpret_cast<uint32_t *>(best1 + Tr::R);
    float *red = reinterpret_cast<float *>(args + (int64_t)T * 64);
    const int bar = 1 + pair;
    u64 cv[Tr::NB][Tr::RT / 2];
    load_pair_values<K>(p.values, pt, cv);
    for (int t = pt; t < T; t += 64) xs[t] = __ldg(p.X + row * (int64_t)T + t);
    const bool has_start = p.start != nullptr;
    const int start = has_start ? (int)(p.start[row] & (kStates - 1)) : 0;
    init_best_pair<K>(best0, pt, has_start, start);
    pair_sync(bar);
    float *bin = best0, *bout = best1;
    for (int t = 1; t < T; ++t) {
        uint32_t words[Tr::WORDS];
        acs_pair<K>(bin, bout, xs[t - 1], pt, cv, words);
        args[(int64_t)t * 64 + pt] = words[0];
        pair_sync(bar);
        float *tmp = bin;
        bin = bout;
        bout = tmp;
    }
    const int fs = final_argmin_pair<K>(bin, xs[T - 1], pt, bar, cv, red);
    if (pt >= 32) return;  // the first warp walks the path (broadcast reads), lane 0 writes it
    int64_t *out = p.states + row * (int64_t)T;
    int s = fs;
    if (pt == 0) out[T - 1] = s;
    for (int t = T - 1; t > 0; --t) {
        const int r = s >> K;
        s = decode_choice<K>(args + (int64_t)t * 64, r) * Tr::R + r;
        if (pt == 0) out[t - 1] = s;
    }
}

// Shared memory of one pair: x (padded to 16 bytes), two best buffers of R floats, T x 64 back-pointer words, 4 words.
size_t pair_long_bytes(int T, int k) {
    const size_t R = (size_t)1 << (kL - k);
    const size_t b = (size_t)(T + 3) / 4 * 16 + 2 * R * sizeof(float) + (size_t)T * 64 * sizeof(uint32_t) + 16;
    return (b + 15) / 16 * 16;
}

__global__ void __launch_bounds__(128) viterbi_pair_long_kernel(VitParams p, int k, int64_t pair_bytes) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int warp = threadIdx.x >> 5, pair = warp >> 1, pt = (warp & 1) * 32 + (threadIdx.x & 31);
    const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 64) + pair;
    if (row >= p.rows) return;  // both warps of the pair leave together: no barrier of this pair is pending
    unsigned char *base = smem + pair * pair_bytes;
    switch (k) {
        case 1: viterbi_pair_long<1>(p, row, pair, pt, base); break;
        case 2: viterbi_pair_long<2>(p, row, pair, pt, base); break;
        case 3: viterbi_pair_long<3>(p, row, pair, pt, base); break;
        default: viterbi_pair_long<4>(p, row, pair, pt, base); break;
    }
}

// Launches the pair decoder when a pair's shared memory fits (two pairs per CTA when both fit); returns false
// otherwise, leaving the call to the one-warp kernel.
bool launch_pair_long(const VitParams &p, int k, cudaStream_t stream, int *rc) {
    int dev = 0, optin = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    const size_t pb = pair_long_bytes(p.T, k);
    const int pairs = 2 * pb <= (size_t)optin ? 2 : (pb <= (size_t)optin ? 1 : 0);
    if (pairs == 0) return false;
    const size_t smem = pairs * pb;
    *rc = LAMQ_OK;
    const cudaError_t e = smem_limit_once((const void *)viterbi_pair_long_kernel, optin);
    if (e != cudaSuccess) {
        set_error("lamq_viterbi: %s", cudaGetErrorString(e));
        *rc = LAMQ_ERR_CUDA;
        return true;
    }
    const int64_t grid = (p.rows + pairs - 1) / pairs;
    viterbi_pair_long_kernel<<<(unsigned)grid, 64 * pairs, smem, stream>>>(p, k, (int64_t)pb);
    const cudaError_t le = cudaGetLastError();
    if (le != cudaSuccess) {
        set_error("lamq_viterbi: %s", cudaGetErrorString(le));
        *rc = LAMQ_ERR_CUDA;
    }
    count_launch();
    return true;
}

}  // namespace

}  // namespace lamq

using namespace lamq;

namespace lamq {
namespace {

// ----------------------------------------------------------------------------- trellises of fewer states
//
// L < 12 (BASELINE config 3's synthetic codebooks have 2^(bits+4) states: L = 5..8; L up to 11 is served): one warp
// per sequence, the 2^L costs of the step before and the 2^(L−k) best values in shared memory, lane l handling states
// l, l + 32, … . Each step takes best_t[r] = min_h cost_{t−1}[h·R + r] (the smallest h on ties, as torch.min) with its
// h stored as a byte per r in the workspace (T x R bytes per sequence), then cost_t[s] = best_t[s >> k] + (x_t − C[s])²
// with the subtraction, the square and the sum each rounded by itself in fp32, as the reference's tensor ops; the
// final state is the first minimum (torch.argmin), and the path is read back from the stored choices.

constexpr int kSmallWarps = 4;

__global__ void __launch_bounds__(kSmallWarps * 32) viterbi_small_kernel(const float *__restrict__ X, int64_t rows,
                                                                           int T, const float *__restrict__ values,
                                                                           int L, int k, const int64_t *start,
                                                                           int64_t *states, uint8_t *back) {
    extern __shared__ __align__(16) float sm[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = 1 << L, R = 1 << (L - k), NB = 1 << k;
    float *C = sm;                                   // S table values (shared by the CTA)
    float *cost = sm + S + warp * (S + R);           // this warp's S costs
    float *best = cost + S;                          // and R best values
    for (int i = threadIdx.x; i < S; i += blockDim.x) C[i] = values[i];
    __syncthreads();
    const int64_t row = (int64_t)blockIdx.x * kSmallWarps + warp;
    if (row >= rows) return;
    const float *x = X + row * (int64_t)T;
    uint8_t *bk = back + row * (int64_t)T * R;
    const float inf = __int_as_float(0x7f800000);
    const float x0 = __ldg(x);
    const bool has_start = start != nullptr;
    const int st0 = has_start ? (int)(start[row] & (S - 1)) : 0;
    for (int s = lane; s < S; s += 32) {
        const float d = __fsub_rn(x0, C[s]);
        const float c = __fmul_rn(d, d);
        // with a start state, only its successors ((start << k) | b) & mask are reachable at the first entry
        cost[s] = (!has_start || (s >> k) == (st0 & (R - 1))) ? c : inf;
    }
    __syncwarp();
    for (int t = 1; t < T; ++t) {
        const float xt = __ldg(x + t);
        for (int r = lane; r < R; r += 32) {
            float m = cost[r];
            int hb = 0;
            for (int h = 1; h < NB; ++h) {
                const float v = cost[h * R + r];
                if (v < m) {
                    m = v;
                    hb = h;
                }
            }
            best[r] = m;
            bk[(int64_t)t * R + r] = (uint8_t)hb;
        }
        __syncwarp();
        for (int s = lane; s < S; s += 32) {
            const float d = __fsub_rn(xt, C[s]);
            cost[s] = __fadd_rn(best[s >> k], __fmul_rn(d, d));
        }
        __syncwarp();
    }
    // the first state of minimum final cost (states visited in increasing order per lane, then the lanes merged)
    float m = inf;
    int ms = 0x7fffffff;
    for (int s = lane; s < S; s += 32) {
        const float v = cost[s];
        if (v < m) {
            m = v;
            ms = s;
        }
    }
    for (int off = 16; off > 0; off >>= 1) {
        const float om = __shfl_xor_sync(0xffffffffu, m, off);
        const int os = __shfl_xor_sync(0xffffffffu, ms, off);
        if (om < m || (om == m && os < ms)) {
            m = om;
            ms = os;
        }
    }
    __syncwarp();
    if (lane == 0) {
        int64_t *out = states + row * (int64_t)T;
        int sc = ms;
        out[T - 1] = sc;
        for (int t = T - 1; t > 0; --t) {
            const int r = sc >> k;
            sc = (int)bk[(int64_t)t * R + r] * R + r;
            out[t - 1] = sc;
        }
    }
}

// Back-pointer bytes of the one-warp kernel for sequences longer than kShortT (32 words of 8 bytes per entry), or
// SIZE_MAX when rows x T x 256 does not fit a size_t.
size_t backptr_bytes(int64_t rows, int T) {
    if (rows <= 0 || T <= kShortT) return 0;
    const size_t per_row = (size_t)T * 32 * sizeof(unsigned long long);
    if ((size_t)rows > SIZE_MAX / per_row) return SIZE_MAX;
    return (size_t)rows * per_row;
}

// Whether the warp-pair decoder takes sequences of T entries on the current device (its back-pointers then live in
// shared memory and no workspace is read).
bool pair_long_fits(int T, int k) {
    int dev = 0, optin = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    if (cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess) return false;
    return pair_long_bytes(T, k) <= (size_t)optin;
}

// The one-warp kernel's shared memory: 8 warps x (two best buffers + 32 steps of back-pointers). Raised once per
// device to the larger of its two sizes, so calls on other host threads never lower it under a pending launch.
constexpr int kVitSmemMax = kVitWarps * (2 * 2048 * (int)sizeof(float) + kShortT * 32 * 8);

int launch_viterbi_warp(const VitParams &p, int k, cudaStream_t stream, const char *fn) {
    const size_t per_warp = 2 * 2048 * sizeof(float) + (p.gargs ? 0 : (size_t)kShortT * 32 * 8);
    const size_t smem = kVitWarps * per_warp;
    const cudaError_t e = smem_limit_once((const void *)viterbi_kernel, kVitSmemMax);
    if (e != cudaSuccess) {
        set_error("%s: %s", fn, cudaGetErrorString(e));
        return LAMQ_ERR_CUDA;
    }
    const int64_t grid = (p.rows + kVitWarps - 1) / kVitWarps;
    LAMQ_REQUIRE(grid <= INT_MAX, "%s: %lld sequences exceed the launch grid", fn, (long long)p.rows);
    viterbi_kernel<<<(unsigned)grid, kVitWarps * 32, smem, stream>>>(p, k);
    LAMQ_CHECK_LAUNCH(fn);
    return LAMQ_OK;
}

}  // namespace
}  // namespace lamq

extern "C" size_t lamq_viterbi_workspace_size(int64_t rows, int T, int L, int k) {
    if (L >= 2 && L < kL && k >= 1 && k < L) {  // fewer states: a byte per r per step
        if (rows <= 0 || T <= 0) return 0;
        const size_t per = (size_t)T << (L - k);
        return (size_t)rows > SIZE_MAX / per ? SIZE_MAX : (size_t)rows * per;
    }
    if (rows <= 0 || T <= kShortT) return 0;
    if (k >= 1 && k <= 4 && pair_long_fits(T, k)) return 0;  // the pair decoder keeps its back-pointers on chip
    return backptr_bytes(rows, T);
}

extern "C" int lamq_viterbi(const float *X, int64_t rows, int T, const float *values, int L, int k,
                            const int64_t *start, int64_t *states, void *workspace, size_t workspace_bytes,
                            lamq_stream_t stream) {
    LAMQ_REQUIRE(L >= 2 && L <= kL, "lamq_viterbi: L must be 2..12 (got %d)", L);
    LAMQ_REQUIRE(k >= 1 && k <= 4 && k < L, "lamq_viterbi: k must be 1..4 and below L (got %d)", k);
    LAMQ_REQUIRE(rows >= 0 && T >= 0, "lamq_viterbi: negative shape");
    if (rows == 0 || T == 0) return LAMQ_OK;
    LAMQ_REQUIRE(X && values && states, "lamq_viterbi: null pointer");
    if (L < kL) {
        const size_t need = lamq_viterbi_workspace_size(rows, T, L, k);
        LAMQ_REQUIRE(need != SIZE_MAX && workspace_bytes >= need && workspace != nullptr,
                     "lamq_viterbi: workspace of %zu bytes needed, %zu given", need, workspace_bytes);
        const int64_t grid = (rows + kSmallWarps - 1) / kSmallWarps;
        LAMQ_REQUIRE(grid <= INT_MAX, "lamq_viterbi: %lld sequences exceed the launch grid", (long long)rows);
        const size_t smem = ((size_t)1 << L) * sizeof(float) +
                            (size_t)kSmallWarps * (((size_t)1 << L) + ((size_t)1 << (L - k))) * sizeof(float);
        const cudaError_t e = smem_limit_once((const void *)viterbi_small_kernel,
                                              (int)((1 << 11) * 4 + kSmallWarps * ((1 << 11) + (1 << 10)) * 4));
        if (e != cudaSuccess) {
            set_error("lamq_viterbi: %s", cudaGetErrorString(e));
            return LAMQ_ERR_CUDA;
        }
        viterbi_small_kernel<<<(unsigned)grid, kSmallWarps * 32, smem, (cudaStream_t)stream>>>(
            X, rows, T, values, L, k, start, states, reinterpret_cast<uint8_t *>(workspace));
        LAMQ_CHECK_LAUNCH("lamq_viterbi (fewer states)");
        return LAMQ_OK;
    }
    if (T > kShortT && pair_long_fits(T, k)) {
        LAMQ_REQUIRE((rows + 1) / 2 <= INT_MAX, "lamq_viterbi: %lld sequences exceed the launch grid", (long long)rows);
        VitParams p{X, rows, T, values, start, states, nullptr};
        int rc = LAMQ_OK;
        if (launch_pair_long(p, k, (cudaStream_t)stream, &rc)) return rc;
    }
    const size_t need = backptr_bytes(rows, T);
    LAMQ_REQUIRE(need != SIZE_MAX, "lamq_viterbi: %lld sequences of %d entries overflow the workspace size",
                 (long long)rows, T);
    LAMQ_REQUIRE(workspace_bytes >= need && (need == 0 || workspace != nullptr),
                 "lamq_viterbi: workspace of %zu bytes needed, %zu given", need, workspace_bytes);
    VitParams p{X, rows, T, values, start, states,
                need ? reinterpret_cast<unsigned long long *>(workspace) : nullptr};
    return launch_viterbi_warp(p, k, (cudaStream_t)stream, "lamq_viterbi");
}

// ----------------------------------------------------------------------------- allocation-free variant
//
// Some callers cannot allocate device memory at all: a host application that hands every byte of the device to its
// own memory pool and forbids libraries from calling cudaMalloc, or a foreign-language binding (cgo, JNI, N-API)
// that has no device allocator of its own to carve a workspace from. lamq_viterbi_noalloc serves them: it decodes
// exactly as lamq_viterbi does, but keeps the back-pointers of long sequences in the array below, which is part of
// the library's device image (every GPU that loads the library holds these 32 MiB until the process exits).
//
// The array's name in host code is only a host-side stand-in for the symbol, never a device address, so the host
// looks the real address up with cudaGetSymbolAddress once per device (with that device current) and passes it to
// the kernel. Every call on a device shares the one array and it keeps whatever the last call left in it; nothing in
// it needs to start at zero, because each back-pointer word the traceback reads was written earlier in the same call.
// Two calls whose kernels overlap on the GPU (on different streams, say) would race on the array.

namespace lamq {
namespace {

constexpr size_t kNoAllocScratchBytes = LAMQ_VITERBI_NOALLOC_SCRATCH_BYTES;
static __device__ __align__(256) unsigned long long g_noalloc_backptr[kNoAllocScratchBytes / sizeof(unsigned long long)];

constexpr int kMaxDevices = 64;
static std::mutex g_noalloc_mu;
static unsigned long long *g_noalloc_addr[kMaxDevices] = {};

// The device address of g_noalloc_backptr on the current device, looked up on the first call per device.
int noalloc_scratch(unsigned long long **out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        set_error("lamq_viterbi_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
        return LAMQ_ERR_CUDA;
    }
    if (dev < 0 || dev >= kMaxDevices) {
        set_error("lamq_viterbi_noalloc: device %d beyond the %d this library tracks", dev, kMaxDevices);
        return LAMQ_ERR_INVALID;
    }
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (g_noalloc_addr[dev] == nullptr) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_backptr);
        if (e != cudaSuccess || p == nullptr) {
            set_error("lamq_viterbi_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
            return LAMQ_ERR_CUDA;
        }
        g_noalloc_addr[dev] = reinterpret_cast<unsigned long long *>(p);
    }
    *out = g_noalloc_addr[dev];
    return LAMQ_OK;
}

}  // namespace
}  // namespace lamq

extern "C" int lamq_viterbi_noalloc(const float *X, int64_t rows, int T, const float *values, int L, int k,
                                    const int64_t *start, int64_t *states, lamq_stream_t stream) {
    LAMQ_REQUIRE(L == kL, "lamq_viterbi_noalloc: only L = 12 is supported (got %d)", L);
    LAMQ_REQUIRE(k >= 1 && k <= 4, "lamq_viterbi_noalloc: k must be 1..4 (got %d)", k);
    LAMQ_REQUIRE(rows >= 0 && T >= 0, "lamq_viterbi_noalloc: negative shape");
    if (rows == 0 || T == 0) return LAMQ_OK;
    // rows x T is bounded before it is multiplied, so the size check below cannot be passed by a wrapped product
    const size_t max_entries = kNoAllocScratchBytes / (32 * 8);
    LAMQ_REQUIRE(T <= kShortT || (size_t)rows <= max_entries / (size_t)T,
                 "lamq_viterbi_noalloc: %lld sequences of %d entries need more back-pointers than the built-in %zu "
                 "bytes (rows x T at most %zu for T > 32); use lamq_viterbi with a workspace",
                 (long long)rows, T, kNoAllocScratchBytes, max_entries);
    const size_t need = backptr_bytes(rows, T);
    LAMQ_REQUIRE(X && values && states, "lamq_viterbi_noalloc: null pointer");
    unsigned long long *scratch = nullptr;
    if (need != 0) {
        const int st = noalloc_scratch(&scratch);
        if (st != LAMQ_OK) return st;
    }
    VitParams p{X, rows, T, values, start, states, need ? scratch : nullptr};
    return launch_viterbi_warp(p, k, (cudaStream_t)stream, "lamq_viterbi_noalloc");
}
