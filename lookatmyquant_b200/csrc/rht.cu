// Randomized Hadamard transforms applied through their Kronecker factors, in fp64.
//
// Reference: opgraph/codes.py:97-132 builds R = hadamard(n)·diag(s) = (A ⊗ B)/√n·diag(s) as a dense n × n matrix
// (A Sylvester, B Sylvester or Paley, entries ±1) and applies it with dense products: X = W·R_inᵀ (codes.py:430),
// Hr = R_in·H·R_inᵀ (codes.py:439), W_q = (S ⊙ V)·R_in (frame.py Net.matrix). Here a row v of length n = a·b, viewed
// as an a × b matrix V, is transformed as (A ⊗ B)·vec(V) = vec(A·V·Bᵀ): b² + a² signed additions per a·b entries
// instead of n² multiply-adds (9728 = 64 · 152: 216 per entry instead of 9728).
//
// One CTA transforms one row in shared memory, in place: phase 1 (one warp per row p of V) forms Z = V·Beᵀ, phase 2
// (one warp per column q) forms Y = Ae·Z; each lane keeps the sign bits of the factor rows it produces in registers.
// A factor that is a natural-order Sylvester matrix (found on the device from its sign bits: every A here, and B when
// n is a power of four) is applied by fast Walsh–Hadamard butterflies instead, log2(order) additions per element
// (64 → 6 at n = 9728; 128 → 7 at 2560; both factors at 4096).
// Fewer than kSplitRows rows (a decode step's few input vectors) are spread over many CTAs instead (the split form).
// The general form computed is y = scale · post ⊙ ((Ae ⊗ Be)·(pre ⊙ v)), so R (Ae = A, Be = B, pre = s) and Rᵀ
// (Ae = Aᵀ, Be = Bᵀ, post = s) are both one pass.
#include <cuda_bf16.h>

#include "lamq_common.cuh"

namespace lamq {

namespace {

constexpr int kRhtThreads = 256;
constexpr int kMaxFactor = 256;  // largest factor order supported (words of sign bits per factor row: 8)

struct RhtParams {
    const double *in;
    int64_t ldi;
    double *out;
    int64_t ldo;
    int64_t rows;
    int a, b;
    const uint32_t *abits;  // a x wa words: bit p' of row p set when Ae[p][p'] = -1
    const uint32_t *bbits;  // b x wb words
    int wa, wb;
    const double *pre, *post;  // n signs or null
    double scale;
};

// acc[c] (output index lane + 32c) += Σ_k sign(bits[c], k) · src[k·stride], k < len; bits[c][w] holds the signs of
// k in [32w, 32w + 32) for the output this lane owns (bit set: negative).
template <int NC>
__device__ __forceinline__ void signed_sums(const double *__restrict__ src, int stride, int len,
                                            const uint32_t (&bits)[NC][NC > 0 ? 8 : 8], double (&acc)[NC]) {
#pragma unroll
    for (int w = 0; w < 8; ++w) {
        if (32 * w >= len) break;
        uint32_t bw[NC];
#pragma unroll
        for (int c = 0; c < NC; ++c) bw[c] = bits[c][w];
        const int lim = min(32, len - 32 * w);
        if (lim == 32) {
#pragma unroll
            for (int bit = 0; bit < 32; ++bit) {
                const long long v = __double_as_longlong(src[(32 * w + bit) * stride]);
#pragma unroll
                for (int c = 0; c < NC; ++c)
                    acc[c] += __longlong_as_double(v ^ ((long long)((bw[c] >> bit) & 1u) << 63));
            }
        } else {
            for (int bit = 0; bit < lim; ++bit) {
                const long long v = __double_as_longlong(src[(32 * w + bit) * stride]);
#pragma unroll
                for (int c = 0; c < NC; ++c)
                    acc[c] += __longlong_as_double(v ^ ((long long)((bw[c] >> bit) & 1u) << 63));
            }
        }
    }
}

// Whether a factor's sign bits are the natural-order Sylvester matrix H[i][j] = (-1)^popcount(i & j) of a power-of-
// two order (every A of codes.hadamard_factors, and B when n is a power of four): checked by the whole CTA.
__device__ __forceinline__ bool sylvester_factor(const uint32_t *__restrict__ bits, int order, int words) {
    bool ok = (order & (order - 1)) == 0;
    for (int e = threadIdx.x; ok && e < order * words; e += blockDim.x) {
        const int r = e / words, w = e - r * words;
        uint32_t want = 0u;
        for (int k = 0; k < 32 && 32 * w + k < order; ++k) want |= (uint32_t)(__popc(r & (32 * w + k)) & 1) << k;
        ok = bits[e] == want;
    }
    return __syncthreads_and(ok) != 0;
}

// x ← H·x for a Sylvester H of order `order` (a power of two), x spread over the warp as x[c] = element lane + 32c:
// the fast Walsh–Hadamard butterflies, log2(order) additions per element instead of `order` signed ones.
template <int NC>
__device__ __forceinline__ void fwht_warp(double (&x)[NC], int order, int lane) {
    for (int h = 1; h < order && h < 32; h <<= 1) {
#pragma unroll
        for (int c = 0; c < NC; ++c) {
            const double v = __shfl_xor_sync(0xffffffffu, x[c], h);
            x[c] = (lane & h) ? __dsub_rn(v, x[c]) : __dadd_rn(x[c], v);
        }
    }
#pragma unroll
    for (int hc = 1; hc < NC; hc <<= 1) {
        if (32 * hc >= order) break;
#pragma unroll
        for (int c = 0; c < NC; ++c) {
            if (c & hc) continue;
            const double u = x[c], v = x[c + hc];
            x[c] = __dadd_rn(u, v);
            x[c + hc] = __dsub_rn(u, v);
        }
    }
}

// NA = ceil(a/32), NB = ceil(b/32): output chunks per lane (and sign words per factor row) of the two phases.
template <int NA, int NB>
__global__ void __launch_bounds__(kRhtThreads) rht_rows_kernel(RhtParams p) {
    extern __shared__ __align__(16) double sv[];
    const int n = p.a * p.b;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = kRhtThreads / 32;
    const bool fast_a = sylvester_factor(p.abits, p.a, p.wa), fast_b = sylvester_factor(p.bbits, p.b, p.wb);
    for (int64_t row = blockIdx.x; row < p.rows; row += gridDim.x) {
        const double *src = p.in + row * p.ldi;
#pragma unroll 8
        for (int e = threadIdx.x; e < n; e += kRhtThreads) sv[e] = p.pre ? src[e] * p.pre[e] : src[e];
        __syncthreads();
        // phase 1: Z[pr][q] = Σ_q' Be[q][q'] · V[pr][q'], a warp per row pr of V, lanes over q
        if (fast_b) {
            for (int pr = warp; pr < p.a; pr += nwarps) {
                double x[NB];
#pragma unroll
                for (int c = 0; c < NB; ++c) x[c] = (lane + 32 * c < p.b) ? sv[pr * p.b + lane + 32 * c] : 0.0;
                fwht_warp<NB>(x, p.b, lane);
#pragma unroll
                for (int c = 0; c < NB; ++c)
                    if (lane + 32 * c < p.b) sv[pr * p.b + lane + 32 * c] = x[c];
            }
        } else {
            uint32_t bits[NB][8];
#pragma unroll
            for (int c = 0; c < NB; ++c) {
                const int q = lane + 32 * c;
#pragma unroll
                for (int w = 0; w < 8; ++w) bits[c][w] = (q < p.b && w < p.wb) ? __ldg(p.bbits + q * p.wb + w) : 0u;
            }
            for (int pr = warp; pr < p.a; pr += nwarps) {
                double acc[NB];
#pragma unroll
                for (int c = 0; c < NB; ++c) acc[c] = 0.0;
                signed_sums<NB>(sv + pr * p.b, 1, p.b, bits, acc);
                __syncwarp();
#pragma unroll
                for (int c = 0; c < NB; ++c) {
                    const int q = lane + 32 * c;
                    if (q < p.b) sv[pr * p.b + q] = acc[c];
                }
                __syncwarp();
            }
        }
        __syncthreads();
        // phase 2: Y[pr][q] = Σ_p' Ae[pr][p'] · Z[p'][q], a warp per column q, lanes over pr
        if (fast_a) {
            for (int q = warp; q < p.b; q += nwarps) {
                double x[NA];
#pragma unroll
                for (int c = 0; c < NA; ++c) x[c] = (lane + 32 * c < p.a) ? sv[(lane + 32 * c) * p.b + q] : 0.0;
                fwht_warp<NA>(x, p.a, lane);
#pragma unroll
                for (int c = 0; c < NA; ++c)
                    if (lane + 32 * c < p.a) sv[(lane + 32 * c) * p.b + q] = x[c];
            }
        } else {
            uint32_t bits[NA][8];
#pragma unroll
            for (int c = 0; c < NA; ++c) {
                const int pr = lane + 32 * c;
#pragma unroll
                for (int w = 0; w < 8; ++w) bits[c][w] = (pr < p.a && w < p.wa) ? __ldg(p.abits + pr * p.wa + w) : 0u;
            }
            for (int q = warp; q < p.b; q += nwarps) {
                double acc[NA];
#pragma unroll
                for (int c = 0; c < NA; ++c) acc[c] = 0.0;
                signed_sums<NA>(sv + q, p.b, p.a, bits, acc);
                __syncwarp();
#pragma unroll
                for (int c = 0; c < NA; ++c) {
                    const int pr = lane + 32 * c;
                    if (pr < p.a) sv[pr * p.b + q] = acc[c];
                }
                __syncwarp();
            }
        }
        __syncthreads();
        double *dst = p.out + row * p.ldo;
#pragma unroll 8
        for (int e = threadIdx.x; e < n; e += kRhtThreads) {
            const double y = sv[e] * p.scale;
            dst[e] = p.post ? y * p.post[e] : y;
        }
        __syncthreads();
    }
}

// The split form, for a few rows: one CTA per row leaves most SMs idle and runs a row's a·b·(a + b) additions on one
// SM, so each row is spread over many CTAs in two launches instead. Row pr of Z = V·Beᵀ depends on row pr of V only,
// and column q of Y = Ae·Z on column q of Z only, so rht_split_rows_kernel writes kSplitWarps rows of Z per CTA into
// `out` and rht_split_cols_kernel turns kSplitWarps columns of Z per CTA into Y in place: the CTAs of a launch share
// no data and no scratch is needed. The sums run in the same order as in rht_rows_kernel, so the results are equal.
constexpr int kSplitWarps = 8;
constexpr int64_t kSplitRows = 128;  // fewer rows than this take the split form

template <int NB>
__global__ void __launch_bounds__(kSplitWarps * 32) rht_split_rows_kernel(RhtParams p) {
    extern __shared__ __align__(16) double sz[];  // kSplitWarps rows of V, b each
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int slices = (p.a + kSplitWarps - 1) / kSplitWarps;
    const int64_t row = blockIdx.x / slices;
    const int pr0 = (int)(blockIdx.x % slices) * kSplitWarps;
    const int nr = min(kSplitWarps, p.a - pr0);
    const int64_t off = (int64_t)pr0 * p.b;
    const double *src = p.in + row * p.ldi + off;
    for (int e = threadIdx.x; e < nr * p.b; e += blockDim.x) sz[e] = p.pre ? src[e] * p.pre[off + e] : src[e];
    __syncthreads();
    const bool fast = sylvester_factor(p.bbits, p.b, p.wb);  // the whole CTA, before any warp leaves
    if (warp >= nr) return;
    double *dst = p.out + row * p.ldo + off + (int64_t)warp * p.b;
    if (fast) {  // the same butterflies as rht_rows_kernel, so the two forms stay equal
        double x[NB];
#pragma unroll
        for (int c = 0; c < NB; ++c) x[c] = (lane + 32 * c < p.b) ? sz[warp * p.b + lane + 32 * c] : 0.0;
        fwht_warp<NB>(x, p.b, lane);
#pragma unroll
        for (int c = 0; c < NB; ++c)
            if (lane + 32 * c < p.b) dst[lane + 32 * c] = x[c];
        return;
    }
    uint32_t bits[NB][8];
#pragma unroll
    for (int c = 0; c < NB; ++c) {
        const int q = lane + 32 * c;
#pragma unroll
        for (int w = 0; w < 8; ++w) bits[c][w] = (q < p.b && w < p.wb) ? __ldg(p.bbits + q * p.wb + w) : 0u;
    }
    double acc[NB];
#pragma unroll
    for (int c = 0; c < NB; ++c) acc[c] = 0.0;
    signed_sums<NB>(sz + warp * p.b, 1, p.b, bits, acc);
#pragma unroll
    for (int c = 0; c < NB; ++c) {
        const int q = lane + 32 * c;
        if (q < p.b) dst[q] = acc[c];
    }
}

template <int NA>
__global__ void __launch_bounds__(kSplitWarps * 32) rht_split_cols_kernel(RhtParams p) {
    extern __shared__ __align__(16) double sz[];  // kSplitWarps columns of Z, a each, at a stride of a + 1
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int slices = (p.b + kSplitWarps - 1) / kSplitWarps;
    const int64_t row = blockIdx.x / slices;
    const int q0 = (int)(blockIdx.x % slices) * kSplitWarps;
    const int nq = min(kSplitWarps, p.b - q0);
    const int ld = p.a + 1;
    double *Z = p.out + row * p.ldo;
    for (int e = threadIdx.x; e < nq * p.a; e += blockDim.x) {  // consecutive threads: consecutive columns of a row
        const int pr = e / nq, w = e - pr * nq;
        sz[w * ld + pr] = Z[(int64_t)pr * p.b + q0 + w];
    }
    __syncthreads();
    const bool fast = sylvester_factor(p.abits, p.a, p.wa);  // the whole CTA, before any warp leaves
    if (warp >= nq) return;
    const int q = q0 + warp;
    if (fast) {  // the same butterflies as rht_rows_kernel, so the two forms stay equal
        double x[NA];
#pragma unroll
        for (int c = 0; c < NA; ++c) x[c] = (lane + 32 * c < p.a) ? sz[warp * ld + lane + 32 * c] : 0.0;
        fwht_warp<NA>(x, p.a, lane);
#pragma unroll
        for (int c = 0; c < NA; ++c) {
            const int pr = lane + 32 * c;
            if (pr < p.a) {
                const int64_t e = (int64_t)pr * p.b + q;
                const double y = x[c] * p.scale;
                Z[e] = p.post ? y * p.post[e] : y;
            }
        }
        return;
    }
    uint32_t bits[NA][8];
#pragma unroll
    for (int c = 0; c < NA; ++c) {
        const int pr = lane + 32 * c;
#pragma unroll
        for (int w = 0; w < 8; ++w) bits[c][w] = (pr < p.a && w < p.wa) ? __ldg(p.abits + pr * p.wa + w) : 0u;
    }
    double acc[NA];
#pragma unroll
    for (int c = 0; c < NA; ++c) acc[c] = 0.0;
    signed_sums<NA>(sz + warp * ld, 1, p.a, bits, acc);
#pragma unroll
    for (int c = 0; c < NA; ++c) {
        const int pr = lane + 32 * c;
        if (pr < p.a) {
            const int64_t e = (int64_t)pr * p.b + q;
            const double y = acc[c] * p.scale;
            Z[e] = p.post ? y * p.post[e] : y;
        }
    }
}

// ---- activations: the same transform in fp32 for many rows, reading bf16/fp32/fp64 and writing bf16 or fp32
//
// The product's inputs and the probed piece's activations go to a bf16 tensor-core operand, so fp32 sums (at most
// a + b = 216 terms of ±1·x) are more than enough; fp32 values take half the shared memory (more rows in flight per
// SM) and the fp32 pipe adds twice as fast as the fp64 one.

template <int NC>
__device__ __forceinline__ void signed_sums_f32(const float *__restrict__ src, int stride, int len,
                                                const uint32_t (&bits)[NC][8], float (&acc)[NC]) {
#pragma unroll
    for (int w = 0; w < 8; ++w) {
        if (32 * w >= len) break;
        uint32_t bw[NC];
#pragma unroll
        for (int c = 0; c < NC; ++c) bw[c] = bits[c][w];
        const int lim = min(32, len - 32 * w);
        if (lim == 32) {
#pragma unroll
            for (int bit = 0; bit < 32; ++bit) {
                const uint32_t v = __float_as_uint(src[(32 * w + bit) * stride]);
#pragma unroll
                for (int c = 0; c < NC; ++c) acc[c] += __uint_as_float(v ^ (((bw[c] >> bit) & 1u) << 31));
            }
        } else {
            for (int bit = 0; bit < lim; ++bit) {
                const uint32_t v = __float_as_uint(src[(32 * w + bit) * stride]);
#pragma unroll
                for (int c = 0; c < NC; ++c) acc[c] += __uint_as_float(v ^ (((bw[c] >> bit) & 1u) << 31));
            }
        }
    }
}

struct RhtActParams {
    const void *in;
    int in_dtype;
    int64_t ldi;
    void *out;
    int out_dtype;
    int64_t ldo;
    int64_t rows;
    int a, b;
    const uint32_t *abits, *bbits;
    int wa, wb;
    const double *pre, *post;  // n signs (±1) or null
    float scale;
};

__device__ __forceinline__ float load_act(const void *p, int dtype, int64_t e) {
    if (dtype == LAMQ_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(p)[e]);
    if (dtype == LAMQ_F32) return reinterpret_cast<const float *>(p)[e];
    return (float)reinterpret_cast<const double *>(p)[e];
}

template <int NA, int NB>
__global__ void __launch_bounds__(kRhtThreads, 2) rht_rows_act_kernel(RhtActParams p) {
    extern __shared__ __align__(16) float svf[];
    const int n = p.a * p.b;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = kRhtThreads / 32;
    for (int64_t row = blockIdx.x; row < p.rows; row += gridDim.x) {
        const int64_t base = row * p.ldi;
#pragma unroll 8
        for (int e = threadIdx.x; e < n; e += kRhtThreads) {
            const float v = load_act(p.in, p.in_dtype, base + e);
            svf[e] = p.pre ? (p.pre[e] < 0 ? -v : v) : v;
        }
        __syncthreads();
        {  // the sign words are loaded per phase (cached): both phases' in registers would halve the resident CTAs
        uint32_t bbits[NB][8];
#pragma unroll
        for (int c = 0; c < NB; ++c) {
            const int q = lane + 32 * c;
#pragma unroll
            for (int w = 0; w < 8; ++w) bbits[c][w] = (q < p.b && w < p.wb) ? __ldg(p.bbits + q * p.wb + w) : 0u;
        }
        for (int pr = warp; pr < p.a; pr += nwarps) {  // Z[pr][q] = Σ_q' Be[q][q']·V[pr][q']
            float acc[NB];
#pragma unroll
            for (int c = 0; c < NB; ++c) acc[c] = 0.f;
            signed_sums_f32<NB>(svf + pr * p.b, 1, p.b, bbits, acc);
            __syncwarp();
#pragma unroll
            for (int c = 0; c < NB; ++c) {
                const int q = lane + 32 * c;
                if (q < p.b) svf[pr * p.b + q] = acc[c];
            }
            __syncwarp();
        }
        }
        __syncthreads();
        {
        uint32_t abits[NA][8];
#pragma unroll
        for (int c = 0; c < NA; ++c) {
            const int pr = lane + 32 * c;
#pragma unroll
            for (int w = 0; w < 8; ++w) abits[c][w] = (pr < p.a && w < p.wa) ? __ldg(p.abits + pr * p.wa + w) : 0u;
        }
        for (int q = warp; q < p.b; q += nwarps) {  // Y[pr][q] = Σ_p' Ae[pr][p']·Z[p'][q]
            float acc[NA];
#pragma unroll
            for (int c = 0; c < NA; ++c) acc[c] = 0.f;
            signed_sums_f32<NA>(svf + q, p.b, p.a, abits, acc);
            __syncwarp();
#pragma unroll
            for (int c = 0; c < NA; ++c) {
                const int pr = lane + 32 * c;
                if (pr < p.a) svf[pr * p.b + q] = acc[c];
            }
            __syncwarp();
        }
        }
        __syncthreads();
        const int64_t obase = row * p.ldo;
#pragma unroll 8
        for (int e = threadIdx.x; e < n; e += kRhtThreads) {
            float y = svf[e] * p.scale;
            if (p.post && p.post[e] < 0) y = -y;
            if (p.out_dtype == LAMQ_BF16)
                reinterpret_cast<__nv_bfloat16 *>(p.out)[obase + e] = __float2bfloat16_rn(y);
            else
                reinterpret_cast<float *>(p.out)[obase + e] = y;
        }
        __syncthreads();
    }
}

template <int NA, int NB>
int launch_rht_act(const RhtActParams &p, cudaStream_t stream) {
    const size_t smem = (size_t)p.a * p.b * sizeof(float);
    const cudaError_t e = smem_limit_once((const void *)rht_rows_act_kernel<NA, NB>, 100 * 1024);
    if (e != cudaSuccess) {
        set_error("lamq_rht_rows_act: %s", cudaGetErrorString(e));
        return LAMQ_ERR_CUDA;
    }
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t grid = p.rows < (int64_t)sms * 8 ? p.rows : (int64_t)sms * 8;
    rht_rows_act_kernel<NA, NB><<<(unsigned)grid, kRhtThreads, smem, stream>>>(p);
    LAMQ_CHECK_LAUNCH("lamq_rht_rows_act");
    return LAMQ_OK;
}

constexpr int kTile = 32;

__global__ void transpose_kernel(const double *__restrict__ in, int64_t ldi, double *__restrict__ out, int64_t ldo,
                                 int rows, int cols) {
    __shared__ double tile[kTile][kTile + 1];
    const int bx = blockIdx.x * kTile, by = blockIdx.y * kTile;
    for (int y = threadIdx.y; y < kTile; y += blockDim.y) {
        const int r = by + y, c = bx + threadIdx.x;
        if (r < rows && c < cols) tile[y][threadIdx.x] = in[(int64_t)r * ldi + c];
    }
    __syncthreads();
    for (int y = threadIdx.y; y < kTile; y += blockDim.y) {
        const int r = bx + y, c = by + threadIdx.x;
        if (r < cols && c < rows) out[(int64_t)r * ldo + c] = tile[threadIdx.x][y];
    }
}

template <int NA, int NB>
int launch_rht(const RhtParams &p, cudaStream_t stream) {
    const size_t smem = (size_t)p.a * p.b * sizeof(double);
    cudaError_t e = smem_limit_max_once((const void *)rht_rows_kernel<NA, NB>);
    if (e != cudaSuccess) {
        set_error("lamq_rht_rows: %s", cudaGetErrorString(e));
        return LAMQ_ERR_CUDA;
    }
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t grid = p.rows < (int64_t)sms * 8 ? p.rows : (int64_t)sms * 8;
    rht_rows_kernel<NA, NB><<<(unsigned)grid, kRhtThreads, smem, stream>>>(p);
    LAMQ_CHECK_LAUNCH("lamq_rht_rows");
    return LAMQ_OK;
}

template <int NA, int NB>
int launch_rht_split(const RhtParams &p, cudaStream_t stream) {
    const int64_t sa = (p.a + kSplitWarps - 1) / kSplitWarps, sb = (p.b + kSplitWarps - 1) / kSplitWarps;
    rht_split_rows_kernel<NB><<<(unsigned)(p.rows * sa), kSplitWarps * 32, (size_t)kSplitWarps * p.b * sizeof(double),
                                stream>>>(p);
    LAMQ_CHECK_LAUNCH("lamq_rht_rows (rows of V)");
    rht_split_cols_kernel<NA><<<(unsigned)(p.rows * sb), kSplitWarps * 32,
                                (size_t)kSplitWarps * (p.a + 1) * sizeof(double), stream>>>(p);
    LAMQ_CHECK_LAUNCH("lamq_rht_rows (columns of Z)");
    return LAMQ_OK;
}

}  // namespace

}  // namespace lamq

using namespace lamq;

extern "C" int lamq_rht_rows(const double *in, int64_t ldi, double *out, int64_t ldo, int64_t rows, int a, int b,
                             const uint32_t *abits, const uint32_t *bbits, const double *pre, const double *post,
                             double scale, lamq_stream_t stream) {
    LAMQ_REQUIRE(rows >= 0 && a >= 1 && b >= 1 && a <= kMaxFactor && b <= kMaxFactor,
                 "lamq_rht_rows: factor orders must be 1..%d", kMaxFactor);
    if (rows == 0) return LAMQ_OK;
    LAMQ_REQUIRE(in && out && abits && bbits, "lamq_rht_rows: null pointer");
    LAMQ_REQUIRE(ldi >= (int64_t)a * b && ldo >= (int64_t)a * b, "lamq_rht_rows: leading dimension below n");
    LAMQ_REQUIRE((size_t)a * b * sizeof(double) <= 200 * 1024, "lamq_rht_rows: n = %d too large for one CTA", a * b);
    RhtParams p{in, ldi, out, ldo, rows, a, b, abits, bbits, (a + 31) / 32, (b + 31) / 32, pre, post, scale};
    const int wa = p.wa, wb = p.wb;
    cudaStream_t s = (cudaStream_t)stream;
    // the output chunks per lane are template parameters so the sums and sign words stay in registers
    const int na = wa <= 1 ? 1 : wa <= 2 ? 2 : wa <= 4 ? 4 : 8;
    const int nb = wb;
#define LAMQ_RHT_CASE(NA_, NB_) \
    if (na == NA_ && nb == NB_)                                                                     \
        return rows < kSplitRows ? launch_rht_split<NA_, NB_>(p, s) : launch_rht<NA_, NB_>(p, s);
#define LAMQ_RHT_ROW(NA_) \
    LAMQ_RHT_CASE(NA_, 1) LAMQ_RHT_CASE(NA_, 2) LAMQ_RHT_CASE(NA_, 3) LAMQ_RHT_CASE(NA_, 4) \
    LAMQ_RHT_CASE(NA_, 5) LAMQ_RHT_CASE(NA_, 6) LAMQ_RHT_CASE(NA_, 7) LAMQ_RHT_CASE(NA_, 8)
    LAMQ_RHT_ROW(1) LAMQ_RHT_ROW(2) LAMQ_RHT_ROW(4) LAMQ_RHT_ROW(8)
#undef LAMQ_RHT_ROW
#undef LAMQ_RHT_CASE
    set_error("lamq_rht_rows: unsupported factor orders %d x %d", a, b);
    return LAMQ_ERR_INVALID;
}

extern "C" int lamq_transpose_f64(const double *in, int64_t ldi, double *out, int64_t ldo, int rows, int cols,
                                  lamq_stream_t stream) {
    LAMQ_REQUIRE(rows >= 0 && cols >= 0, "lamq_transpose_f64: negative shape");
    if (rows == 0 || cols == 0) return LAMQ_OK;
    LAMQ_REQUIRE(in && out && in != out, "lamq_transpose_f64: null or aliased pointer");
    dim3 grid((cols + kTile - 1) / kTile, (rows + kTile - 1) / kTile), block(kTile, 8);
    transpose_kernel<<<grid, block, 0, (cudaStream_t)stream>>>(in, ldi, out, ldo, rows, cols);
    LAMQ_CHECK_LAUNCH("lamq_transpose_f64");
    return LAMQ_OK;
}

extern "C" int lamq_rht_rows_act(const void *in, int in_dtype, int64_t ldi, void *out, int out_dtype, int64_t ldo,
                                 int64_t rows, int a, int b, const uint32_t *abits, const uint32_t *bbits,
                                 const double *pre, const double *post, double scale, lamq_stream_t stream) {
    LAMQ_REQUIRE(rows >= 0 && a >= 1 && b >= 1 && a <= kMaxFactor && b <= kMaxFactor,
                 "lamq_rht_rows_act: factor orders must be 1..%d", kMaxFactor);
    LAMQ_REQUIRE(in_dtype == LAMQ_F32 || in_dtype == LAMQ_BF16 || in_dtype == LAMQ_F64,
                 "lamq_rht_rows_act: input dtype must be LAMQ_F32, LAMQ_BF16 or LAMQ_F64");
    LAMQ_REQUIRE(out_dtype == LAMQ_F32 || out_dtype == LAMQ_BF16,
                 "lamq_rht_rows_act: output dtype must be LAMQ_F32 or LAMQ_BF16");
    if (rows == 0) return LAMQ_OK;
    LAMQ_REQUIRE(in && out && abits && bbits, "lamq_rht_rows_act: null pointer");
    LAMQ_REQUIRE(ldi >= (int64_t)a * b && ldo >= (int64_t)a * b, "lamq_rht_rows_act: leading dimension below n");
    LAMQ_REQUIRE(in != out, "lamq_rht_rows_act: in and out must not alias");
    LAMQ_REQUIRE((size_t)a * b * sizeof(float) <= 100 * 1024, "lamq_rht_rows_act: n = %d too large for one CTA", a * b);
    RhtActParams p{in, in_dtype, ldi, out, out_dtype, ldo, rows, a, b, abits, bbits, (a + 31) / 32, (b + 31) / 32,
                   pre, post, (float)scale};
    const int na = p.wa <= 1 ? 1 : p.wa <= 2 ? 2 : p.wa <= 4 ? 4 : 8;
    const int nb = p.wb;
    cudaStream_t s = (cudaStream_t)stream;
#define LAMQ_RHT_ACT_CASE(NA_, NB_) \
    if (na == NA_ && nb == NB_) return launch_rht_act<NA_, NB_>(p, s);
#define LAMQ_RHT_ACT_ROW(NA_) \
    LAMQ_RHT_ACT_CASE(NA_, 1) LAMQ_RHT_ACT_CASE(NA_, 2) LAMQ_RHT_ACT_CASE(NA_, 3) LAMQ_RHT_ACT_CASE(NA_, 4) \
    LAMQ_RHT_ACT_CASE(NA_, 5) LAMQ_RHT_ACT_CASE(NA_, 6) LAMQ_RHT_ACT_CASE(NA_, 7) LAMQ_RHT_ACT_CASE(NA_, 8)
    LAMQ_RHT_ACT_ROW(1) LAMQ_RHT_ACT_ROW(2) LAMQ_RHT_ACT_ROW(4) LAMQ_RHT_ACT_ROW(8)
#undef LAMQ_RHT_ACT_ROW
#undef LAMQ_RHT_ACT_CASE
    set_error("lamq_rht_rows_act: unsupported factor orders %d x %d", a, b);
    return LAMQ_ERR_INVALID;
}
