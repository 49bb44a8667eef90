// The packed trellis format of opgraph-packed-1 on the device: packing int16 states into the reversed k-bit stream,
// unpacking, decoding rows to weights, and the product of packed rows with input vectors.
//
// Reference: compiler_artifact.py:225-297 (`pack_symbols`, `unpack_symbols`, `valid_path`, `pack_trellis`,
// `unpack_trellis`), :433-442 (`decode_rotated`), and the product kernel of runtime_mlx/fast_q35.py:69-172.
//
// Format. A row of n states with k-bit symbols is padded forward to N = 32·⌈n/32⌉ columns (zero symbols after the
// last real column) and reversed, so symbol p of the stream is the symbol of column N − 1 − p. Symbol p occupies bits
// [p·k, p·k + k) of the row's little-endian bit stream of N·k bits = N/32·k uint32 words. A trellis path from state 0
// has state_j = the L bits of the stream at bit (N − 1 − j)·k (bits past the end read as zero), so every state is
// read straight from the stream, without a walk along the row.
#include <algorithm>

#include "lamq_common.cuh"

namespace lamq {
namespace {

__device__ __forceinline__ uint32_t stream_bits(const uint32_t *__restrict__ row, int wpr, int64_t bit, int width) {
    const int64_t w = bit >> 5;
    const int off = (int)(bit & 31);
    const uint32_t lo = (w < wpr) ? __ldg(row + w) : 0u;
    const uint32_t hi = (w + 1 < wpr) ? __ldg(row + w + 1) : 0u;
    const uint64_t v = ((uint64_t)hi << 32 | lo) >> off;
    return (uint32_t)v & ((1u << width) - 1u);
}

// One thread per output word: gathers the symbols that overlap bits [32w, 32w + 32) of row r and checks the path at
// the columns of those symbols (compiler_artifact.py:261-267).
__global__ void pack_trellis_kernel(const int16_t *__restrict__ states, int64_t lds, int64_t rows, int n, int k, int L,
                                    uint32_t *__restrict__ codes, int *status) {
    const int N = (n + 31) / 32 * 32;
    const int wpr = N / 32 * k;
    const int64_t total = rows * wpr;
    const uint32_t kmask = (1u << k) - 1u, tail = (1u << (L - k)) - 1u;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = e / wpr;
        const int w = (int)(e % wpr);
        const int16_t *srow = states + r * lds;
        uint32_t word = 0;
        bool bad = false;
        const int p0 = (32 * w) / k, p1 = (32 * w + 31) / k;
        for (int p = p0; p <= p1; ++p) {
            const int j = N - 1 - p;
            uint32_t sym = 0;
            if (j < n) {
                const int s = srow[j];
                if (s < 0 || s >= (1 << L)) bad = true;
                if (j == 0) {
                    if (s >= (1 << k)) bad = true;
                } else {
                    const int prev = srow[j - 1];
                    if (((uint32_t)s >> k) != ((uint32_t)prev & tail)) bad = true;
                }
                sym = (uint32_t)s & kmask;
            }
            const int shift = p * k - 32 * w;
            word |= shift >= 0 ? (sym << shift) : (sym >> -shift);
        }
        codes[e] = word;
        if (bad) atomicCAS(status, 0, LAMQ_ERR_NOT_PATH);
    }
}

// state_j of every (row, column); with `table`, out = table[state]·scale[r] (fp32, compiler_artifact.py:440) at row
// map[r] (or r), else the states as int16.
__global__ void unpack_trellis_kernel(const uint32_t *__restrict__ codes, int64_t rows, int n, int k, int L,
                                      int16_t *__restrict__ states, int64_t lds, const float *__restrict__ table,
                                      const float *__restrict__ scales, const uint32_t *__restrict__ map,
                                      float *__restrict__ out, int64_t ldo) {
    const int N = (n + 31) / 32 * 32;
    const int wpr = N / 32 * k;
    const int64_t total = rows * n;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = e / n;
        const int j = (int)(e % n);
        const uint32_t s = stream_bits(codes + r * wpr, wpr, (int64_t)(N - 1 - j) * k, L);
        if (table == nullptr) {
            states[r * lds + j] = (int16_t)s;
        } else {
            const int64_t orow = map ? (int64_t)map[r] : r;
            out[orow * ldo + j] = __fmul_rn(__ldg(table + s), __ldg(scales + r));
        }
    }
}

// y[v][map[r]] = scale[r] · Σ_j table[state_rj] · x[v][j] for NV input vectors. A CTA of 8 warps takes
// kRowsPerCta rows at a time; warp w walks its share of the columns 32 at a time (lane = column): each lane reads the
// one or two stream words that hold its column's state (the warp's 32 columns share k + 1 words, which L1 serves),
// looks the value up in the table (shared memory) and multiplies it into the NV vectors' sums, each x value reused
// across the rows. The warps' partial sums are added in a fixed order through shared memory, so the result is
// deterministic. A persistent grid loads the table once per CTA.
constexpr int kRowsPerCta = 4;
constexpr int kProductWarps = 8;
constexpr int kColumnBlocks = 4;

template <int NV>
__global__ void __launch_bounds__(kProductWarps * 32) trellis_product_kernel(
    const uint32_t *__restrict__ codes, int64_t rows, int n, int k, int L, const float *__restrict__ scales,
    const float *__restrict__ table, const uint32_t *__restrict__ map, const float *__restrict__ x, int64_t ldx,
    float *__restrict__ y, int64_t ldy) {
    __shared__ __align__(16) float tab[4096];
    __shared__ float part[kProductWarps][kRowsPerCta][NV];
    const int nt = 1 << L;
    if ((reinterpret_cast<uintptr_t>(table) & 15) == 0 && nt >= 4) {  // 16-byte loads, all in flight together
#pragma unroll 4
        for (int i = threadIdx.x; i < nt / 4; i += blockDim.x)
            reinterpret_cast<float4 *>(tab)[i] = __ldg(reinterpret_cast<const float4 *>(table) + i);
    } else {
#pragma unroll 16
        for (int i = threadIdx.x; i < nt; i += blockDim.x) tab[i] = __ldg(table + i);
    }
    __syncthreads();
    const int N = (n + 31) / 32 * 32;
    const int wpr = N / 32 * k;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int chunk = (N / 32 + kProductWarps - 1) / kProductWarps * 32;  // columns per warp, a multiple of 32
    const int c0 = warp * chunk, c1 = min(n, c0 + chunk);
    const int64_t groups = (rows + kRowsPerCta - 1) / kRowsPerCta;
    for (int64_t g = blockIdx.x; g < groups; g += gridDim.x) {
        const int64_t r0 = g * kRowsPerCta;
        float acc[kRowsPerCta][NV];
#pragma unroll
        for (int a = 0; a < kRowsPerCta; ++a)
#pragma unroll
            for (int v = 0; v < NV; ++v) acc[a][v] = 0.f;
        // kColumnBlocks blocks of 32 columns per step: their stream words are loaded together, so a warp waits on
        // memory once per step rather than once per block
        for (int j0 = c0; j0 < c1; j0 += 32 * kColumnBlocks) {
            uint32_t st[kColumnBlocks][kRowsPerCta];
#pragma unroll
            for (int u = 0; u < kColumnBlocks; ++u) {
                const int j = j0 + 32 * u + lane;
#pragma unroll
                for (int a = 0; a < kRowsPerCta; ++a) {
                    const int64_t r = min(r0 + a, rows - 1);
                    st[u][a] = (j < c1) ? stream_bits(codes + r * wpr, wpr, (int64_t)(N - 1 - j) * k, L) : 0u;
                }
            }
#pragma unroll
            for (int u = 0; u < kColumnBlocks; ++u) {
                const int j = j0 + 32 * u + lane;
                if (j < c1) {
                    float val[kRowsPerCta];
#pragma unroll
                    for (int a = 0; a < kRowsPerCta; ++a) val[a] = tab[st[u][a]];
#pragma unroll
                    for (int v = 0; v < NV; ++v) {
                        const float xv = __ldg(x + (int64_t)v * ldx + j);
#pragma unroll
                        for (int a = 0; a < kRowsPerCta; ++a) acc[a][v] = fmaf(val[a], xv, acc[a][v]);
                    }
                }
            }
        }
#pragma unroll
        for (int a = 0; a < kRowsPerCta; ++a)
#pragma unroll
            for (int v = 0; v < NV; ++v) {
                float s = acc[a][v];
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
                if (lane == 0) part[warp][a][v] = s;
            }
        __syncthreads();
        for (int e = threadIdx.x; e < kRowsPerCta * NV; e += blockDim.x) {
            const int a = e / NV, v = e % NV;
            const int64_t r = r0 + a;
            if (r < rows) {
                float s = 0.f;
#pragma unroll
                for (int w = 0; w < kProductWarps; ++w) s += part[w][a][v];
                const int64_t orow = map ? (int64_t)map[r] : r;
                y[(int64_t)v * ldy + orow] = s * scales[r];
            }
        }
        __syncthreads();  // part is rewritten by the next rows
    }
}

// The 2^L values of a table into shared memory, 16 bytes a load where the table's alignment allows.
__device__ __forceinline__ void load_table(float *tab, const float *__restrict__ table, int L) {
    const int nt = 1 << L;
    if ((reinterpret_cast<uintptr_t>(table) & 15) == 0 && nt >= 4) {
#pragma unroll 4
        for (int i = threadIdx.x; i < nt / 4; i += blockDim.x)
            reinterpret_cast<float4 *>(tab)[i] = __ldg(reinterpret_cast<const float4 *>(table) + i);
    } else {
#pragma unroll 16
        for (int i = threadIdx.x; i < nt; i += blockDim.x) tab[i] = __ldg(table + i);
    }
}

// The three stream words that hold the states of columns jb .. jb + 7 of rows r0 .. r0 + kRowsPerCta − 1 (rows past
// the end repeat the last row; words past the row's end read as zero), and the bit offset of column jb + 7's state in
// the first word: column jb + i has its state at bit (N − 1 − jb − i)·K, (7 − i)·K above that of column jb + 7.
template <int K>
__device__ __forceinline__ void load_words(const uint32_t *__restrict__ codes, int64_t rows, int wpr, int N,
                                           int64_t r0, int jb, uint32_t (&wv)[kRowsPerCta][3], int &sh0) {
    const int64_t bp = (int64_t)(N - 1 - (jb + 7)) * K;
    const int64_t w0 = bp >> 5;
    sh0 = (int)(bp & 31);
#pragma unroll
    for (int a = 0; a < kRowsPerCta; ++a) {
        const uint32_t *row = codes + min(r0 + a, rows - 1) * wpr;
#pragma unroll
        for (int q = 0; q < 3; ++q) wv[a][q] = (w0 + q < wpr) ? __ldg(row + w0 + q) : 0u;
    }
}

// The product for symbol widths K = 1..4, a lane owning 8 consecutive columns: their 8 states lie within
// 7K + L <= 40 bits of the row's stream, so three words loaded once give all 8 (a 64-bit window, then a funnel shift
// by a constant each),
// and the 8 input values arrive as two float4 loads per vector. The CTA's 8 warps take the 256-column blocks of rows
// r0 .. r0 + kRowsPerCta − 1 in turn, and their partial sums are added in a fixed order through shared memory, so a
// row's result does not depend on which launch or CTA computed it. Every thread of the CTA calls this; it ends with
// a barrier, after which `tab` and `part` may be rewritten.
template <int NV, int K>
__device__ __forceinline__ void product8_rows(const uint32_t *__restrict__ codes, int64_t rows, int n, uint32_t smask,
                                              const float *__restrict__ scales, const float *tab,
                                              const uint32_t *__restrict__ map, const float *__restrict__ x,
                                              int64_t ldx, int xvec, float *__restrict__ y, int64_t ldy, int64_t r0,
                                              float (*part)[kRowsPerCta][NV]) {
    const int N = (n + 31) / 32 * 32;
    const int wpr = N / 32 * K;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nblk = (n + 255) / 256;
    float acc[kRowsPerCta][NV];
#pragma unroll
    for (int a = 0; a < kRowsPerCta; ++a)
#pragma unroll
        for (int v = 0; v < NV; ++v) acc[a][v] = 0.f;
    for (int blk = warp; blk < nblk; blk += kProductWarps) {
        const int jb = blk * 256 + lane * 8;  // this lane's first column
        if (jb < n) {
            uint32_t wv[kRowsPerCta][3];
            int sh0;
            load_words<K>(codes, rows, wpr, N, r0, jb, wv, sh0);
            // bits [sh0, sh0 + 64) of each row's stream: column jb + i's state starts (7 − i)·K <= 28 bits in, and
            // 28 + L <= 40, so every state is one funnel shift by a constant
            uint32_t lo[kRowsPerCta], hi[kRowsPerCta];
#pragma unroll
            for (int a = 0; a < kRowsPerCta; ++a) {
                lo[a] = __funnelshift_r(wv[a][0], wv[a][1], sh0);
                hi[a] = __funnelshift_r(wv[a][1], wv[a][2], sh0);
            }
            const bool full = xvec && jb + 8 <= n;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                float xv[NV][4];
#pragma unroll
                for (int v = 0; v < NV; ++v) {
                    const float *xp = x + (int64_t)v * ldx + jb + 4 * h;
                    if (full) {
                        const float4 t = __ldg(reinterpret_cast<const float4 *>(xp));
                        xv[v][0] = t.x; xv[v][1] = t.y; xv[v][2] = t.z; xv[v][3] = t.w;
                    } else {
#pragma unroll
                        for (int i = 0; i < 4; ++i) xv[v][i] = (jb + 4 * h + i < n) ? __ldg(xp + i) : 0.f;
                    }
                }
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    constexpr int kLast = 7 * K;
                    const int r = kLast - (4 * h + i) * K;  // a constant after unrolling
#pragma unroll
                    for (int a = 0; a < kRowsPerCta; ++a) {
                        const float val = tab[__funnelshift_r(lo[a], hi[a], r) & smask];
#pragma unroll
                        for (int v = 0; v < NV; ++v) acc[a][v] = fmaf(val, xv[v][i], acc[a][v]);
                    }
                }
            }
        }
    }
#pragma unroll
    for (int a = 0; a < kRowsPerCta; ++a)
#pragma unroll
        for (int v = 0; v < NV; ++v) {
            float s = acc[a][v];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            if (lane == 0) part[warp][a][v] = s;
        }
    __syncthreads();
    for (int e = threadIdx.x; e < kRowsPerCta * NV; e += blockDim.x) {
        const int a = e / NV, v = e % NV;
        const int64_t r = r0 + a;
        if (r < rows) {
            float s = 0.f;
#pragma unroll
            for (int w = 0; w < kProductWarps; ++w) s += part[w][a][v];
            const int64_t orow = map ? (int64_t)map[r] : r;
            y[(int64_t)v * ldy + orow] = s * scales[r];
        }
    }
    __syncthreads();  // part (and, between matrices, tab) is rewritten next
}

// One packed matrix (one row group of one width) times NV vectors; a persistent grid loads the table once per CTA.
template <int NV, int K>
__global__ void __launch_bounds__(kProductWarps * 32) trellis_product8_kernel(
    const uint32_t *__restrict__ codes, int64_t rows, int n, int L, const float *__restrict__ scales,
    const float *__restrict__ table, const uint32_t *__restrict__ map, const float *__restrict__ x, int64_t ldx,
    int xvec, float *__restrict__ y, int64_t ldy) {
    __shared__ __align__(16) float tab[4096];
    __shared__ float part[kProductWarps][kRowsPerCta][NV];
    load_table(tab, table, L);
    __syncthreads();
    const uint32_t smask = (1u << L) - 1u;
    const int64_t groups = (rows + kRowsPerCta - 1) / kRowsPerCta;
    for (int64_t g = blockIdx.x; g < groups; g += gridDim.x)
        product8_rows<NV, K>(codes, rows, n, smask, scales, tab, map, x, ldx, xvec, y, ldy, g * kRowsPerCta, part);
}

// Several packed matrices that read the same input vectors (the row groups of a stage's matrices, each of its own
// width, table, scales and output), in one launch: their kRowsPerCta-row units are numbered one after another and
// every CTA takes a contiguous share of them, so it crosses few matrix boundaries and loads few tables. A row's
// result is the same as from trellis_product8_kernel, bit for bit (the same body and reduction order).
constexpr int kMaxProductGroups = 32;

struct ProductGroups {
    const uint32_t *codes[kMaxProductGroups];
    const float *scales[kMaxProductGroups];
    const float *table[kMaxProductGroups];
    const uint32_t *map[kMaxProductGroups];
    float *y[kMaxProductGroups];
    int64_t rows[kMaxProductGroups];
    int64_t ldy[kMaxProductGroups];
    int64_t first[kMaxProductGroups + 1];  // the first unit of each matrix; first[ng] = all units
    int k[kMaxProductGroups];
    int L[kMaxProductGroups];
    int ng;
};

template <int NV>
__global__ void __launch_bounds__(kProductWarps * 32) trellis_product_groups_kernel(
    const __grid_constant__ ProductGroups p, int n, const float *__restrict__ x, int64_t ldx, int xvec) {
    __shared__ __align__(16) float tab[4096];
    __shared__ float part[kProductWarps][kRowsPerCta][NV];
    const int64_t total = p.first[p.ng];
    const int64_t u0 = total * blockIdx.x / gridDim.x, u1 = total * (blockIdx.x + 1) / gridDim.x;
    int i = 0, loaded = -1;
    for (int64_t u = u0; u < u1; ++u) {
        while (u >= p.first[i + 1]) ++i;  // u < total, so i stays below ng; empty matrices are skipped
        if (i != loaded) {  // the previous rows' product ended with a barrier: nobody reads tab now
            load_table(tab, p.table[i], p.L[i]);
            __syncthreads();
            loaded = i;
        }
        const uint32_t smask = (1u << p.L[i]) - 1u;
        const int64_t r0 = (u - p.first[i]) * kRowsPerCta;
        switch (p.k[i]) {
            case 1: product8_rows<NV, 1>(p.codes[i], p.rows[i], n, smask, p.scales[i], tab, p.map[i], x, ldx, xvec,
                                         p.y[i], p.ldy[i], r0, part); break;
            case 2: product8_rows<NV, 2>(p.codes[i], p.rows[i], n, smask, p.scales[i], tab, p.map[i], x, ldx, xvec,
                                         p.y[i], p.ldy[i], r0, part); break;
            case 3: product8_rows<NV, 3>(p.codes[i], p.rows[i], n, smask, p.scales[i], tab, p.map[i], x, ldx, xvec,
                                         p.y[i], p.ldy[i], r0, part); break;
            default: product8_rows<NV, 4>(p.codes[i], p.rows[i], n, smask, p.scales[i], tab, p.map[i], x, ldx, xvec,
                                          p.y[i], p.ldy[i], r0, part); break;
        }
    }
}

int grid_for(int64_t work, int threads) {
    return (int)std::min<int64_t>((work + threads - 1) / threads, 148 * 32);
}

// The CTAs of a product kernel that are resident together on the whole GPU (registers and shared memory decide how
// many fit on an SM): the persistent grids are no larger, so no CTA waits for a second wave with a full share of rows.
int resident_grid(const void *kernel) {
    int dev = 0, sms = 148, per = 1;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        sms = 148;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, kernel, kProductWarps * 32, 0) != cudaSuccess || per < 1)
        per = 1;
    return sms * per;
}

template <int NV, int K>
void launch_product8(int64_t units, const uint32_t *codes, int64_t rows, int n, int L, const float *scales,
                     const float *table, const uint32_t *map, const float *x, int64_t ldx, int xvec, float *y,
                     int64_t ldy, cudaStream_t s) {
    const int grid = (int)std::min<int64_t>(units, resident_grid((const void *)trellis_product8_kernel<NV, K>));
    trellis_product8_kernel<NV, K><<<grid, kProductWarps * 32, 0, s>>>(codes, rows, n, L, scales, table, map, x, ldx,
                                                                       xvec, y, ldy);
}

template <int NV>
void launch_product(const uint32_t *codes, int64_t rows, int n, int k, int L, const float *scales, const float *table,
                    const uint32_t *map, const float *x, int64_t ldx, float *y, int64_t ldy, cudaStream_t s) {
    const int64_t units = (rows + kRowsPerCta - 1) / kRowsPerCta;
    const int xvec = ((uintptr_t)x % 16 == 0 && ldx % 4 == 0) ? 1 : 0;
    switch (k) {  // the widths of the trellis codes; wider symbols take the general kernel
        case 1: launch_product8<NV, 1>(units, codes, rows, n, L, scales, table, map, x, ldx, xvec, y, ldy, s); break;
        case 2: launch_product8<NV, 2>(units, codes, rows, n, L, scales, table, map, x, ldx, xvec, y, ldy, s); break;
        case 3: launch_product8<NV, 3>(units, codes, rows, n, L, scales, table, map, x, ldx, xvec, y, ldy, s); break;
        case 4: launch_product8<NV, 4>(units, codes, rows, n, L, scales, table, map, x, ldx, xvec, y, ldy, s); break;
        default: {
            const int grid = (int)std::min<int64_t>(units, 148 * 6);
            trellis_product_kernel<NV><<<grid, kProductWarps * 32, 0, s>>>(codes, rows, n, k, L, scales, table, map, x,
                                                                           ldx, y, ldy);
        }
    }
}

template <int NV>
void launch_groups(const ProductGroups &p, int n, const float *x, int64_t ldx, int xvec, cudaStream_t s) {
    const int grid =
        (int)std::min<int64_t>(p.first[p.ng], resident_grid((const void *)trellis_product_groups_kernel<NV>));
    trellis_product_groups_kernel<NV><<<grid, kProductWarps * 32, 0, s>>>(p, n, x, ldx, xvec);
}

}  // namespace
}  // namespace lamq

using namespace lamq;

// Symbols of 1-8 bits (pack_symbols' range) and states of more bits than a symbol, at most 12 (a table of <= 4096).
#define LAMQ_CHECK_FORMAT(fn)                                                                                   \
    LAMQ_REQUIRE(rows >= 0 && n > 0, fn ": bad shape");                                                         \
    LAMQ_REQUIRE(k >= 1 && k <= 8 && L > k && L <= 12, fn ": unsupported widths (k %d, L %d)", k, L)

extern "C" int64_t lamq_trellis_words_per_row(int n, int k) { return n <= 0 || k <= 0 ? 0 : (int64_t)(n + 31) / 32 * k; }

extern "C" int lamq_pack_trellis(const int16_t *states, int64_t lds, int64_t rows, int n, int k, int L, uint32_t *codes,
                                 int *status, lamq_stream_t stream) {
    LAMQ_CHECK_FORMAT("lamq_pack_trellis");
    LAMQ_REQUIRE(lds >= n, "lamq_pack_trellis: leading dimension below n");
    if (rows == 0) return LAMQ_OK;
    LAMQ_REQUIRE(states && codes && status, "lamq_pack_trellis: null pointer");
    const int64_t work = rows * lamq_trellis_words_per_row(n, k);
    pack_trellis_kernel<<<grid_for(work, 256), 256, 0, (cudaStream_t)stream>>>(states, lds, rows, n, k, L, codes, status);
    LAMQ_CHECK_LAUNCH("lamq_pack_trellis");
    return LAMQ_OK;
}

extern "C" int lamq_unpack_trellis(const uint32_t *codes, int64_t rows, int n, int k, int L, int16_t *states,
                                   int64_t lds, lamq_stream_t stream) {
    LAMQ_CHECK_FORMAT("lamq_unpack_trellis");
    LAMQ_REQUIRE(lds >= n, "lamq_unpack_trellis: leading dimension below n");
    if (rows == 0) return LAMQ_OK;
    LAMQ_REQUIRE(codes && states, "lamq_unpack_trellis: null pointer");
    unpack_trellis_kernel<<<grid_for(rows * n, 256), 256, 0, (cudaStream_t)stream>>>(
        codes, rows, n, k, L, states, lds, nullptr, nullptr, nullptr, nullptr, 0);
    LAMQ_CHECK_LAUNCH("lamq_unpack_trellis");
    return LAMQ_OK;
}

extern "C" int lamq_decode_trellis(const uint32_t *codes, int64_t rows, int n, int k, int L, const float *scales,
                                   const float *table, const uint32_t *map, float *out, int64_t ldo,
                                   lamq_stream_t stream) {
    LAMQ_CHECK_FORMAT("lamq_decode_trellis");
    LAMQ_REQUIRE(ldo >= n, "lamq_decode_trellis: leading dimension below n");
    if (rows == 0) return LAMQ_OK;
    LAMQ_REQUIRE(codes && scales && table && out, "lamq_decode_trellis: null pointer");
    unpack_trellis_kernel<<<grid_for(rows * n, 256), 256, 0, (cudaStream_t)stream>>>(
        codes, rows, n, k, L, nullptr, 0, table, scales, map, out, ldo);
    LAMQ_CHECK_LAUNCH("lamq_decode_trellis");
    return LAMQ_OK;
}

extern "C" int lamq_trellis_product(const uint32_t *codes, int64_t rows, int n, int k, int L, const float *scales,
                                    const float *table, const uint32_t *map, const float *x, int64_t ldx, int nvec,
                                    float *y, int64_t ldy, lamq_stream_t stream) {
    LAMQ_CHECK_FORMAT("lamq_trellis_product");
    LAMQ_REQUIRE(nvec >= 0 && ldx >= n, "lamq_trellis_product: bad vector shape");
    if (rows == 0 || nvec == 0) return LAMQ_OK;
    LAMQ_REQUIRE(codes && scales && table && x && y, "lamq_trellis_product: null pointer");
    // each vector's output row holds every group row (map or not): shorter rows would overlap the next vector's
    LAMQ_REQUIRE(nvec <= 1 || ldy >= rows, "lamq_trellis_product: ldy %lld below the group's %lld rows",
                 (long long)ldy, (long long)rows);
    cudaStream_t s = (cudaStream_t)stream;
    for (int v = 0; v < nvec;) {
        const int left = nvec - v;
        const float *xv = x + (int64_t)v * ldx;
        float *yv = y + (int64_t)v * ldy;
        if (left >= 16) launch_product<16>(codes, rows, n, k, L, scales, table, map, xv, ldx, yv, ldy, s), v += 16;
        else if (left >= 8) launch_product<8>(codes, rows, n, k, L, scales, table, map, xv, ldx, yv, ldy, s), v += 8;
        else if (left >= 4) launch_product<4>(codes, rows, n, k, L, scales, table, map, xv, ldx, yv, ldy, s), v += 4;
        else if (left >= 2) launch_product<2>(codes, rows, n, k, L, scales, table, map, xv, ldx, yv, ldy, s), v += 2;
        else launch_product<1>(codes, rows, n, k, L, scales, table, map, xv, ldx, yv, ldy, s), v += 1;
        LAMQ_CHECK_LAUNCH("lamq_trellis_product");
    }
    return LAMQ_OK;
}

static_assert(sizeof(lamq_product_group) == 64, "lamq_product_group is 64 bytes in the C ABI");

extern "C" int lamq_trellis_product_groups(const lamq_product_group *groups, int ngroups, int n, const float *x,
                                           int64_t ldx, int nvec, lamq_stream_t stream) {
    LAMQ_REQUIRE(ngroups >= 0 && n > 0 && nvec >= 0 && ldx >= n, "lamq_trellis_product_groups: bad shape");
    if (ngroups == 0 || nvec == 0) return LAMQ_OK;
    LAMQ_REQUIRE(groups && x, "lamq_trellis_product_groups: null pointer");
    for (int i = 0; i < ngroups; ++i) {
        const lamq_product_group &g = groups[i];
        LAMQ_REQUIRE(g.rows >= 0, "lamq_trellis_product_groups: group %d has %lld rows", i, (long long)g.rows);
        LAMQ_REQUIRE(g.k >= 1 && g.k <= 4 && g.L > g.k && g.L <= 12,
                     "lamq_trellis_product_groups: group %d: widths k in 1..4 and L in k+1..12 (k %d, L %d)", i, g.k,
                     g.L);
        LAMQ_REQUIRE(g.rows == 0 || (g.codes && g.scales && g.table && g.y),
                     "lamq_trellis_product_groups: group %d: null pointer", i);
        LAMQ_REQUIRE(nvec <= 1 || g.ldy >= g.rows,
                     "lamq_trellis_product_groups: group %d: ldy %lld below its %lld rows", i, (long long)g.ldy,
                     (long long)g.rows);
    }
    cudaStream_t s = (cudaStream_t)stream;
    const int xvec = ((uintptr_t)x % 16 == 0 && ldx % 4 == 0) ? 1 : 0;
    for (int b = 0; b < ngroups; b += kMaxProductGroups) {
        ProductGroups p{};
        int64_t units = 0;
        int ng = 0;
        for (int i = b; i < std::min(ngroups, b + kMaxProductGroups); ++i, ++ng) {
            const lamq_product_group &g = groups[i];
            p.codes[ng] = g.codes;
            p.scales[ng] = g.scales;
            p.table[ng] = g.table;
            p.map[ng] = g.map;
            p.y[ng] = g.y;
            p.rows[ng] = g.rows;
            p.ldy[ng] = g.ldy;
            p.k[ng] = g.k;
            p.L[ng] = g.L;
            p.first[ng] = units;
            units += (g.rows + kRowsPerCta - 1) / kRowsPerCta;
        }
        p.first[ng] = units;
        p.ng = ng;
        if (units == 0) continue;
        // at most 8 vectors a launch: 16 take 255 registers a thread and one CTA per SM, and two 8-vector passes
        // over the (L2-resident) codes of a layer were faster than one 16-vector pass (0.44 against 0.50 ms)
        for (int v = 0; v < nvec;) {
            const int left = nvec - v;
            const int nv = left >= 8 ? 8 : left >= 4 ? 4 : left >= 2 ? 2 : 1;
            ProductGroups q = p;
            for (int i = 0; i < ng; ++i) q.y[i] = p.y[i] + (int64_t)v * p.ldy[i];
            const float *xv = x + (int64_t)v * ldx;
            switch (nv) {
                case 8: launch_groups<8>(q, n, xv, ldx, xvec, s); break;
                case 4: launch_groups<4>(q, n, xv, ldx, xvec, s); break;
                case 2: launch_groups<2>(q, n, xv, ldx, xvec, s); break;
                default: launch_groups<1>(q, n, xv, ldx, xvec, s); break;
            }
            LAMQ_CHECK_LAUNCH("lamq_trellis_product_groups");
            v += nv;
        }
    }
    return LAMQ_OK;
}
