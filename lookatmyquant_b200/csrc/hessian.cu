// Token-weighted Hessian (and QEP cross-moment) accumulation on tcgen05 tensor cores.
//
// Reference: quantize.py:1412-1470 (`quantize_stage`): per calibration chunk H += Xᵀ(w⊙X) and D += X_refᵀ(w⊙X) in
// fp32, then H/n_tok and D/n_tok − H as fp64; compiler.py:233-265 (`capture`) is the unweighted form.
//
// The contraction C[j][i] += Σ_t A[t][i]·B[t][j] over tokens t runs as a persistent warp-specialised GEMM:
//   warp 0     one thread issues TMA loads of 64-token tiles of A (128 columns) and B (256 columns) (bf16, row-major
//              tokens × d, so both operands are MN-major in shared memory, 128-byte swizzle) into a 4-stage ring;
//   warp 1     one thread issues tcgen05.mma (M = 128, N = 256, K = 16, bf16 × bf16 → fp32) into one of two TMEM
//              accumulators (the whole 512 columns), releasing each stage with tcgen05.commit;
//   warps 2-9  drain a finished accumulator with tcgen05.ld into an fp32 tile held in their registers (two warps per
//              TMEM lane quadrant, one row of 128 columns per thread, added with round-to-nearest), while the MMA
//              thread fills the other one; at the end of a unit they add the tile into the fp32 d × d accumulator in
//              global memory (coalesced: written transposed).
// The tensor core's own fp32 accumulation truncates (it loses about half an ulp per MMA on average, always towards
// zero), so TMEM only ever accumulates kDrainBlocks × 4 = 64 MMAs (1024 tokens) before it is drained into the
// registers: the bias stays near 2e-6 relative (measured: 2.2e-6 at d = 2560, 262,144 weighted tokens; 1.1e-6 with
// 512-token drains, slower by 6 %), where a whole chunk in TMEM would bias H by more than the 1e-5 bar.
// A work unit is one 128 × 256 output tile over one chunk of tokens. The tiles are listed band by band (bands of about
// 16 row tiles, column by column inside a band) and cut into windows of exactly one tile per CTA; units run window by
// window, chunk by chunk inside a window. So each wave of CTAs computes one window over one chunk: a compact block of
// about 16 × 9 tiles whose CTAs read the same A and B tiles at about the same time and share them through L2. For H
// only tiles that hold a pair i <= j are computed (H is symmetric); the finalize kernel mirrors them.
// From d = 512 on, xtx_pair_kernel (below) computes 256 × 256 tiles on pairs of CTAs (cta_group::2 MMAs): half the
// operand bytes per CTA per flop, a 6-stage ring.
//
// Fixed summation order: inside a full window CTA b computes the window's tile b over every chunk in turn, so each
// element of that tile is added into the accumulator by one thread, chunk after chunk. The last, partial window has
// fewer tiles than CTAs, so a tile's chunks run on several CTAs at once: there each unit stores its tile (times the
// launch's scale) into a scratch slot of its own, and after the launch a reduction adds every element's slots into the
// accumulator in chunk order. Every element's fp32 sum therefore runs in the same order on every run: the statistics,
// and the layer built from them, are bit-reproducible for a given call sequence and GPU.
//
// Token weights: bf16 products are exact in fp32, but w·x is not a bf16 number. So the main pass runs with w = 1
// (A = X, B = X: exact products), and the weighted tokens add Σ_t (w_t − 1)·x_t x_tᵀ in a second pass over only
// those tokens, with (w − 1)·x split into a bf16 pair hi + lo (hi = bf16(y), lo = bf16(y − hi)), which carries y to
// 2⁻¹⁷ relative — the same result as the reference's fp32 w⊙X to well within its fp32 rounding.
#include <cuda.h>
#include <cuda_bf16.h>

#include <algorithm>
#include <mutex>

#include "lamq_common.cuh"
#include "sm100.cuh"

namespace lamq {

namespace {

using namespace sm100;

constexpr int BM = 128, BN = 256, BK = 64;
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;  // 16 KiB: two 64-column boxes of 64 tokens
constexpr int B_BYTES = BN * BK * 2;  // 32 KiB: four boxes
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int HALF_BYTES = 64 * BK * 2;  // one TMA box: 64 columns x 64 tokens = 8 KiB (LBO between MN blocks)
constexpr int kBandTarget = 16;          // row tiles per band (bands are evened out to at most this many)
constexpr int kDrainBlocks = 16;         // 64-token blocks accumulated in TMEM between drains (64 MMAs)
constexpr int kEpiWarps = 8;             // two per TMEM lane quadrant, 128 columns each
constexpr int kThreads = (2 + kEpiWarps) * 32;
constexpr uint32_t kTmemCols = 512;      // two 128 x 256 fp32 accumulators
constexpr size_t kSmemBytes = 1024 + STAGES * STAGE_BYTES + 256;
// The wave gate keeps the CTAs in step: CTA b runs units b, b + G, b + 2G, … (G CTAs), and its producer starts wave w
// only once the producers have issued every load of waves 0 … w − 1. Without it the CTAs drift apart over the
// waves (a CTA that misses in L2 falls behind and then misses more), the CTAs that share an A or B tile no longer
// read it at about the same time, and DRAM re-reads the operands several times over. The gate is a throttle, not a
// correctness condition: a wait longer than kGateTimeoutNs (CTAs not co-resident, a producer that stopped on an
// error) switches the gate off for the rest of the launch.
constexpr unsigned long long kGateTimeoutNs = 20000000ull;
constexpr int kGateSlots = 64;

struct GemmParams {
    float *acc;
    int64_t ldc;
    int d;
    int nti, ntj;           // row tiles (128) and column tiles (256)
    int band;               // row tiles per band
    int64_t ntiles;         // tiles computed
    int win;                // tiles per window (= CTAs)
    int nchunk;
    int kblocks;            // total 64-token blocks
    int kblocks_per_chunk;
    int symmetric;
    int pair;               // tiles of 256 x 256 computed by a pair of CTAs (cta_group::2), else 128 x 256 per CTA
    float scale;            // each unit's tile is added into acc times this
    int64_t units;
    int *status;
    unsigned int *gate;     // units whose loads have all been issued (the wave gate), zeroed before the launch
    float *scratch;         // the last window's units: slot (chunk, tile − last0, CTA of the pair), or null
    int64_t last0;          // the first tile of the last window (tiles from here on go through the scratch)
    int last_tiles;
};

struct Unit {
    int ti, tj, kb0, nkb;
    int64_t tile;  // index in the band raster
    int chunk;
};

// Tiles of column tj inside the band of row tiles [b0, b1). Symmetric C: row tile ti (rows 128·ti..) and column tile
// tj (columns 256·tj..) hold a pair i <= j iff tj >= ti / 2, that is ti < 2·tj + 2.
__device__ __forceinline__ int band_column(int b0, int b1, int tj, const GemmParams &p) {
    // paired tiles are square: row tile ti holds a pair i <= j iff ti <= tj
    return p.symmetric ? max(0, min(b1, p.pair ? tj + 1 : 2 * tj + 2) - b0) : b1 - b0;
}

// The idx-th tile of the band raster (bands top to bottom, columns left to right, rows top to bottom).
__device__ void tile_at(int64_t idx, const GemmParams &p, int &ti, int &tj) {
    for (int b0 = 0; b0 < p.nti; b0 += p.band) {
        const int b1 = min(p.nti, b0 + p.band);
        for (int c = 0; c < p.ntj; ++c) {
            const int n = band_column(b0, b1, c, p);
            if (idx < n) {
                ti = b0 + (int)idx;
                tj = c;
                return;
            }
            idx -= n;
        }
    }
    ti = tj = 0;  // not reached: idx < ntiles
}

// The u-th work unit: windows of p.win consecutive tiles in order, then chunks, then the window's tiles.
__device__ bool unit_at(int64_t u, const GemmParams &p, Unit &out) {
    const int64_t full = p.ntiles / p.win, per_full = (int64_t)p.win * p.nchunk;
    int64_t idx;
    int chunk;
    if (u < full * per_full) {
        const int64_t w = u / per_full, rem = u % per_full;
        chunk = (int)(rem / p.win);
        idx = w * p.win + rem % p.win;
    } else {
        const int64_t last = p.ntiles - full * p.win, rem = u - full * per_full;
        if (last == 0 || rem >= last * p.nchunk) return false;
        chunk = (int)(rem / last);
        idx = full * p.win + rem % last;
    }
    tile_at(idx, p, out.ti, out.tj);
    out.tile = idx;
    out.chunk = chunk;
    out.kb0 = chunk * p.kblocks_per_chunk;
    out.nkb = min(p.kblocks_per_chunk, p.kblocks - out.kb0);
    return true;
}

__device__ __forceinline__ unsigned int ld_relaxed_u32(const unsigned int *p) {
    unsigned int v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ unsigned int ld_acquire_u32(const unsigned int *p) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

constexpr int kSlotFloats = 128 * 256;  // one CTA's part of a unit's tile: 128 rows x 256 columns

// A drain thread's part of a unit's tile (row i_loc of the CTA's 128, columns c0.. c0 + 127 of its 256) into the
// accumulator (atomic adds; one writer per element in a full window) or, in the last window, into the unit's scratch
// slot (column-major within the slot, so a warp's stores are coalesced).
__device__ __forceinline__ void flush_tile(const GemmParams &p, const Unit &U, int rank, int i_loc, int c0,
                                           const float (&tile)[128], int i, int j0) {
    if (p.scratch != nullptr && U.tile >= p.last0) {
        float *slot = p.scratch +
                      (((int64_t)U.chunk * p.last_tiles + (U.tile - p.last0)) * 2 + rank) * kSlotFloats;
#pragma unroll
        for (int c = 0; c < 128; ++c) slot[(int64_t)(c0 + c) * 128 + i_loc] = tile[c] * p.scale;
        return;
    }
    if (i >= p.d) return;
#pragma unroll
    for (int c = 0; c < 128; ++c) {
        const int j = j0 + c;
        if (j < p.d) atomicAdd(p.acc + (int64_t)j * p.ldc + i, p.scale == 1.0f ? tile[c] : tile[c] * p.scale);
    }
}

// 32 lanes x 32 bits, 32 consecutive columns: thread t of the warp gets lane (base lane + t).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}

__global__ void __launch_bounds__(kThreads, 1)
    xtx_kernel(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapB, GemmParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + STAGES * STAGE_BYTES);
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 2 * STAGES + 5);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + STAGES);
    const uint32_t tfull0 = smem_u32(bars + 2 * STAGES), tempty0 = smem_u32(bars + 2 * STAGES + 2);
    const uint32_t drain = smem_u32(bars + 2 * STAGES + 4);

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(tfull0 + 8 * a, 1);
            mbar_init(tempty0 + 8 * a, kEpiWarps * 32);
        }
        mbar_init(drain, 1);
        fence_mbar_init();
        prefetch_tmap(&mapA);
        prefetch_tmap(&mapB);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_holder), kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;

    if (warp == 0) {
        if (lane == 0) {  // ---- TMA producer
            int stage = 0;
            uint32_t phase = 0;
            int64_t issued = 0;
            bool ok = true, gate = p.gate != nullptr;
            int64_t wave = 0;
            for (int64_t u = blockIdx.x; ok && u < p.units; u += gridDim.x, ++wave) {
                Unit U;
                if (!unit_at(u, p, U)) break;
                if (gate && wave > 0) {
                    const unsigned int target = (unsigned int)(wave * gridDim.x);
                    const unsigned long long t0 = globaltimer();
                    while (ld_relaxed_u32(p.gate) < target) {
                        if (globaltimer() - t0 > kGateTimeoutNs) {
                            gate = false;
                            break;
                        }
                        __nanosleep(256);
                    }
                }
                for (int kb = 0; kb < U.nkb; ++kb) {
                    if (!mbar_wait(empty0 + 8 * stage, phase ^ 1, p.status)) {
                        ok = false;
                        break;
                    }
                    const uint32_t fb = full0 + 8 * stage;
                    mbar_expect_tx(fb, STAGE_BYTES);
                    const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES), sb = sa + A_BYTES;
                    const int t = (U.kb0 + kb) * BK;
                    tma_load_2d(sa, &mapA, U.ti * BM, t, fb);
                    tma_load_2d(sa + HALF_BYTES, &mapA, U.ti * BM + 64, t, fb);
#pragma unroll
                    for (int q = 0; q < BN / 64; ++q) tma_load_2d(sb + q * HALF_BYTES, &mapB, U.tj * BN + 64 * q, t, fb);
                    ++issued;
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (ok && p.gate != nullptr) atomicAdd(p.gate, 1u);
            }
            if (!ok) {  // error path: let the copies already in flight land before the CTA exits
                const int64_t outstanding = issued < STAGES ? issued : STAGES;
                for (int64_t i = issued - outstanding; i < issued; ++i) {
                    const int s = (int)(i % STAGES);
                    const uint32_t ph = (uint32_t)((i / STAGES) & 1);
                    const unsigned long long t0 = globaltimer();
                    while (!mbar_try_wait(full0 + 8 * s, ph) && globaltimer() - t0 < kWaitTimeoutNs) {
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {  // ---- MMA issuer
            const uint32_t idesc = idesc_bf16_f32(BM, BN, true, true);
            int stage = 0;
            uint32_t phase = 0;
            uint32_t uses[2] = {0, 0};
            int acc = 0;
            bool ok = true;
            for (int64_t u = blockIdx.x; ok && u < p.units; u += gridDim.x) {
                Unit U;
                if (!unit_at(u, p, U)) break;
                for (int sub = 0; ok && sub < U.nkb; sub += kDrainBlocks) {
                    if (!mbar_wait(tempty0 + 8 * acc, (uses[acc] & 1) ^ 1, p.status)) {
                        ok = false;
                        break;
                    }
                    ++uses[acc];
                    tc_fence_after();
                    const uint32_t d = tmem + acc * BN;
                    const int kend = min(U.nkb, sub + kDrainBlocks);
                    for (int kb = sub; kb < kend; ++kb) {
                        if (!mbar_wait(full0 + 8 * stage, phase, p.status)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES), sb = sa + A_BYTES;
#pragma unroll
                        for (int kk = 0; kk < BK / 16; ++kk) {
                            // 16 tokens = two 8-row groups of 128 bytes: advance 2 KiB per K step
                            const uint64_t ad = smem_desc_sw128(sa + kk * 2048, HALF_BYTES, 1024);
                            const uint64_t bd = smem_desc_sw128(sb + kk * 2048, HALF_BYTES, 1024);
                            mma_f16_ss(d, ad, bd, idesc, (kb > sub || kk > 0) ? 1u : 0u);
                        }
                        mma_commit(empty0 + 8 * stage);
                        if (++stage == STAGES) {
                            stage = 0;
                            phase ^= 1;
                        }
                    }
                    if (!ok) break;
                    mma_commit(tfull0 + 8 * acc);
                    acc ^= 1;
                }
            }
            // every MMA this thread issued completes before TMEM is released
            mma_commit(drain);
            const unsigned long long t0 = globaltimer();
            while (!mbar_try_wait(drain, 0) && globaltimer() - t0 < kWaitTimeoutNs) {
            }
        }
    } else {  // ---- epilogue: warps 2..9; warp w reads TMEM lanes 32·(w % 4).., columns 128·((w − 2) / 4)..
        const int q = warp & 3, half = (warp - 2) >> 2;
        uint32_t uses[2] = {0, 0};
        int acc = 0;
        for (int64_t u = blockIdx.x; u < p.units; u += gridDim.x) {
            Unit U;
            if (!unit_at(u, p, U)) break;
            float tile[128];
#pragma unroll
            for (int c = 0; c < 128; ++c) tile[c] = 0.f;
            bool ok = true;
            for (int sub = 0; sub < U.nkb; sub += kDrainBlocks) {
                if (!mbar_wait(tfull0 + 8 * acc, uses[acc] & 1, p.status)) {
                    ok = false;
                    break;
                }
                ++uses[acc];
                tc_fence_after();
                const uint32_t tbase = tmem + ((uint32_t)(32 * q) << 16) + acc * BN + 128 * half;
#pragma unroll
                for (int c = 0; c < 128 / 32; ++c) {
                    uint32_t r[32];
                    tmem_ld32(tbase + c * 32, r);
                    tmem_ld_wait();
#pragma unroll
                    for (int e = 0; e < 32; ++e) tile[c * 32 + e] = __fadd_rn(tile[c * 32 + e], __uint_as_float(r[e]));
                }
                tc_fence_before();
                mbar_arrive(tempty0 + 8 * acc);
                acc ^= 1;
            }
            if (!ok) break;
            flush_tile(p, U, 0, 32 * q + lane, 128 * half, tile, U.ti * BM + 32 * q + lane, U.tj * BN + 128 * half);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

// The same contraction with 256 x 256 tiles computed by a pair of CTAs (a cluster of two) with cta_group::2 MMAs
// (M = 256, N = 256, K = 16): each CTA loads its 128 rows of A and its 128 columns of B per 64-token slice (32 KiB
// instead of 48 KiB for a 128 x 256 tile of its own), so a 6-stage ring fits and covers more of the load latency,
// and each CTA's TMEM holds its 128 rows x 256 columns. The even CTA issues the MMAs; both CTAs' loads complete on
// its full barriers; its commits release both CTAs' ring stages and accumulators (multicast commit); both CTAs'
// drain warps release an accumulator on the even CTA's barrier. No TMA multicast: each CTA loads its own halves.
constexpr int PSTAGES = 6;
constexpr int P_A_BYTES = 128 * BK * 2, P_B_BYTES = 128 * BK * 2, P_STAGE_BYTES = P_A_BYTES + P_B_BYTES;
constexpr size_t kPairSmemBytes = 1024 + PSTAGES * P_STAGE_BYTES + 256;
constexpr int kPairBandTarget = 8;

__global__ void __launch_bounds__(kThreads, 1)
    xtx_pair_kernel(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapB, GemmParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + PSTAGES * P_STAGE_BYTES);
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 2 * PSTAGES + 5);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const bool leader = rank == 0;
    const int64_t cluster = blockIdx.x >> 1, nclusters = gridDim.x >> 1;
    const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + PSTAGES);
    const uint32_t tfull0 = smem_u32(bars + 2 * PSTAGES), tempty0 = smem_u32(bars + 2 * PSTAGES + 2);
    const uint32_t drain = smem_u32(bars + 2 * PSTAGES + 4);

    if (threadIdx.x == 0) {
        for (int s = 0; s < PSTAGES; ++s) {
            mbar_init(full0 + 8 * s, 1);   // the even CTA's expect_tx (its full barriers count both CTAs' bytes)
            mbar_init(empty0 + 8 * s, 1);  // the even CTA's multicast commit
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(tfull0 + 8 * a, 1);
            mbar_init(tempty0 + 8 * a, 2 * kEpiWarps * 32);  // both CTAs' drain threads (used on the even CTA)
        }
        mbar_init(drain, 1);
        fence_mbar_init();
        prefetch_tmap(&mapA);
        prefetch_tmap(&mapB);
    }
    if (warp == 1) {  // the same warp in both CTAs allocates the pair's TMEM
        tmem_alloc_pair(smem_u32(tmem_holder), kTmemCols);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync_all();  // both CTAs' barriers exist before either signals the other
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;

    if (warp == 0) {
        if (lane == 0) {  // ---- TMA producer (both CTAs: each loads its own halves)
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true, gate = leader && p.gate != nullptr;
            int64_t wave = 0;
            for (int64_t u = cluster; ok && u < p.units; u += nclusters, ++wave) {
                Unit U;
                if (!unit_at(u, p, U)) break;
                if (gate && wave > 0) {
                    const unsigned int target = (unsigned int)(wave * nclusters);
                    const unsigned long long t0 = globaltimer();
                    while (ld_relaxed_u32(p.gate) < target) {
                        if (globaltimer() - t0 > kGateTimeoutNs) {
                            gate = false;
                            break;
                        }
                        __nanosleep(256);
                    }
                }
                const int ra = U.ti * 256 + 128 * (int)rank, rb = U.tj * 256 + 128 * (int)rank;
                for (int kb = 0; kb < U.nkb; ++kb) {
                    if (!mbar_wait(empty0 + 8 * stage, phase ^ 1, p.status)) {
                        ok = false;
                        break;
                    }
                    if (leader) mbar_expect_tx(full0 + 8 * stage, 2 * P_STAGE_BYTES);
                    const uint32_t fb = map_to_rank(full0 + 8 * stage, 0);
                    const uint32_t sa = smem_u32(smem + stage * P_STAGE_BYTES), sb = sa + P_A_BYTES;
                    const int t = (U.kb0 + kb) * BK;
                    tma_load_2d_pair(sa, &mapA, ra, t, fb);
                    tma_load_2d_pair(sa + HALF_BYTES, &mapA, ra + 64, t, fb);
                    tma_load_2d_pair(sb, &mapB, rb, t, fb);
                    tma_load_2d_pair(sb + HALF_BYTES, &mapB, rb + 64, t, fb);
                    if (++stage == PSTAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (ok && gate) atomicAdd(p.gate, 1u);
            }
            if (!ok) __nanosleep(200000);  // error path: the copies in flight land (their barrier is the even CTA's)
        }
    } else if (warp == 1) {
        if (lane == 0 && leader) {  // ---- MMA issuer (the even CTA)
            const uint32_t idesc = idesc_bf16_f32(256, 256, true, true);
            int stage = 0;
            uint32_t phase = 0;
            uint32_t uses[2] = {0, 0};
            int acc = 0;
            bool ok = true;
            for (int64_t u = cluster; ok && u < p.units; u += nclusters) {
                Unit U;
                if (!unit_at(u, p, U)) break;
                for (int sub = 0; ok && sub < U.nkb; sub += kDrainBlocks) {
                    if (!mbar_wait(tempty0 + 8 * acc, (uses[acc] & 1) ^ 1, p.status)) {
                        ok = false;
                        break;
                    }
                    ++uses[acc];
                    tc_fence_after();
                    const uint32_t d = tmem + acc * BN;
                    const int kend = min(U.nkb, sub + kDrainBlocks);
                    for (int kb = sub; kb < kend; ++kb) {
                        if (!mbar_wait(full0 + 8 * stage, phase, p.status)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t sa = smem_u32(smem + stage * P_STAGE_BYTES), sb = sa + P_A_BYTES;
#pragma unroll
                        for (int kk = 0; kk < BK / 16; ++kk) {
                            const uint64_t ad = smem_desc_sw128(sa + kk * 2048, HALF_BYTES, 1024);
                            const uint64_t bd = smem_desc_sw128(sb + kk * 2048, HALF_BYTES, 1024);
                            mma_f16_ss_pair(d, ad, bd, idesc, (kb > sub || kk > 0) ? 1u : 0u);
                        }
                        mma_commit_pair_multicast(empty0 + 8 * stage, 0x3);
                        if (++stage == PSTAGES) {
                            stage = 0;
                            phase ^= 1;
                        }
                    }
                    if (!ok) break;
                    mma_commit_pair_multicast(tfull0 + 8 * acc, 0x3);
                    acc ^= 1;
                }
            }
            // every MMA this thread issued completes before TMEM is released
            mma_commit_pair(drain);
            const unsigned long long t0 = globaltimer();
            while (!mbar_try_wait(drain, 0) && globaltimer() - t0 < kWaitTimeoutNs) {
            }
        }
    } else {  // ---- drain warps (both CTAs): warp w reads TMEM lanes 32·(w % 4).., columns 128·((w − 2) / 4)..
        const int q = warp & 3, half = (warp - 2) >> 2;
        const uint32_t release = leader ? 0u : 1u;  // the peer's threads arrive on the even CTA's barrier
        uint32_t uses[2] = {0, 0};
        int acc = 0;
        for (int64_t u = cluster; u < p.units; u += nclusters) {
            Unit U;
            if (!unit_at(u, p, U)) break;
            float tile[128];
#pragma unroll
            for (int c = 0; c < 128; ++c) tile[c] = 0.f;
            bool ok = true;
            for (int sub = 0; sub < U.nkb; sub += kDrainBlocks) {
                if (!mbar_wait(tfull0 + 8 * acc, uses[acc] & 1, p.status)) {
                    ok = false;
                    break;
                }
                ++uses[acc];
                tc_fence_after();
                const uint32_t tbase = tmem + ((uint32_t)(32 * q) << 16) + acc * BN + 128 * half;
#pragma unroll
                for (int c = 0; c < 128 / 32; ++c) {
                    uint32_t r[32];
                    tmem_ld32(tbase + c * 32, r);
                    tmem_ld_wait();
#pragma unroll
                    for (int e = 0; e < 32; ++e) tile[c * 32 + e] = __fadd_rn(tile[c * 32 + e], __uint_as_float(r[e]));
                }
                tc_fence_before();
                if (release) mbar_arrive_cluster(map_to_rank(tempty0 + 8 * acc, 0));
                else mbar_arrive(tempty0 + 8 * acc);
                acc ^= 1;
            }
            if (!ok) break;
            flush_tile(p, U, (int)rank, 32 * q + lane, 128 * half, tile, U.ti * 256 + 128 * (int)rank + 32 * q + lane,
                       U.tj * BN + 128 * half);
        }
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync_all();  // neither CTA leaves while the pair's MMAs or arrivals may still touch it
    tc_fence_after();
    if (warp == 1) tmem_dealloc_pair(tmem, kTmemCols);
}

// Weighted tokens: out_plain rows r and r + nw hold plain[idx[r]]; out_split row r holds hi and row r + nw holds lo
// of y = (w[idx[r]] − 1)·scaled[idx[r]] (fp32), hi = bf16(y), lo = bf16(y − hi).
__global__ void weighted_split_kernel(const __nv_bfloat16 *__restrict__ scaled, int64_t lds,
                                      const __nv_bfloat16 *__restrict__ plain, int64_t ldp,
                                      const float *__restrict__ w, const int32_t *__restrict__ idx, int64_t nw, int d,
                                      __nv_bfloat16 *__restrict__ out_split, __nv_bfloat16 *__restrict__ out_plain) {
    const int64_t r = blockIdx.x;
    if (r >= nw) return;
    const int64_t t = idx[r];
    const float f = __fsub_rn(w[t], 1.0f);
    for (int c = threadIdx.x; c < d; c += blockDim.x) {
        const float y = __fmul_rn(f, __bfloat162float(scaled[t * lds + c]));
        const __nv_bfloat16 hi = __float2bfloat16_rn(y);
        const __nv_bfloat16 lo = __float2bfloat16_rn(__fsub_rn(y, __bfloat162float(hi)));
        out_split[r * d + c] = hi;
        out_split[(r + nw) * d + c] = lo;
        const __nv_bfloat16 pv = plain[t * ldp + c];
        out_plain[r * d + c] = pv;
        out_plain[(r + nw) * d + c] = pv;
    }
}

// dst row r = src row idx[r] (bf16 rows as 16-byte units; d a multiple of 8).
__global__ void gather_rows_kernel(const uint4 *__restrict__ src, int64_t lds16, const int32_t *__restrict__ idx,
                                   int64_t n, int units, uint4 *__restrict__ dst) {
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n * units; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = e / units;
        const int u = (int)(e % units);
        dst[r * units + u] = src[(int64_t)idx[r] * lds16 + u];
    }
}

// H[r][c] = acc[max][min] / n_tok (the computed triangle, mirrored); D = accD / n_tok − H.
__global__ void finalize_kernel(const float *__restrict__ accH, const float *__restrict__ accD, int64_t lda, int d,
                                double inv_n, double *__restrict__ H, double *__restrict__ D) {
    const int64_t n = (int64_t)d * d;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
        const int r = (int)(e / d), c = (int)(e % d);
        const int hi = r > c ? r : c, lo = r > c ? c : r;
        const double h = (double)accH[(int64_t)hi * lda + lo] * inv_n;
        H[e] = h;
        if (D != nullptr) D[e] = (double)accD[(int64_t)r * lda + c] * inv_n - h;
    }
}

// The last window's slots added into the accumulator in chunk order: block row y = one CTA part (tile, rank) of the
// last window, its threads over the part's 128 x 256 elements.
__global__ void last_window_reduce_kernel(GemmParams p) {
    const int part = blockIdx.y, tl = part >> 1, rank = part & 1;
    if (!p.pair && rank == 1) return;
    __shared__ int tij[2];
    if (threadIdx.x == 0) tile_at(p.last0 + tl, p, tij[0], tij[1]);
    __syncthreads();
    const int ti = tij[0], tj = tij[1];
    const int64_t chunk_stride = (int64_t)p.last_tiles * 2 * kSlotFloats;
    const float *src = p.scratch + (int64_t)part * kSlotFloats;
    for (int loc = blockIdx.x * blockDim.x + threadIdx.x; loc < kSlotFloats; loc += gridDim.x * blockDim.x) {
        const int col = loc >> 7, i_loc = loc & 127;
        const int i = p.pair ? ti * 256 + 128 * rank + i_loc : ti * BM + i_loc;
        const int j = tj * BN + col;
        if (i >= p.d || j >= p.d) continue;
        float *dst = p.acc + (int64_t)j * p.ldc + i;
        float v = *dst;
        for (int c = 0; c < p.nchunk; ++c) v = __fadd_rn(v, src[(int64_t)c * chunk_stride + loc]);
        *dst = v;
    }
}

// ---- host

using EncodeTiled = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                 const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encode_fn() {
    static std::once_flag once;
    static EncodeTiled fn = nullptr;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiled>(p);
    });
    return fn;
}

// Tokens x d bf16 row-major (leading dimension ld elements): boxes of 64 columns x 64 tokens, 128-byte swizzle.
int make_map(CUtensorMap *m, const void *base, int64_t tokens, int d, int64_t ld, const char *who) {
    EncodeTiled enc = encode_fn();
    if (enc == nullptr) {
        set_error("%s: cuTensorMapEncodeTiled is unavailable", who);
        return LAMQ_ERR_CUDA;
    }
    cuuint64_t dims[2] = {(cuuint64_t)d, (cuuint64_t)tokens};
    cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    cuuint32_t box[2] = {64, (cuuint32_t)BK};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("%s: cuTensorMapEncodeTiled failed (%d)", who, (int)r);
        return LAMQ_ERR_INVALID;
    }
    return LAMQ_OK;
}

constexpr int kMaxDevices = 64;
__device__ unsigned int g_gate[kGateSlots];  // one array per device (module globals are per device)
// A wave-gate counter for one launch on the current device: slots are handed out round robin (launches in flight at
// once take different slots) and zeroed on the launch's stream.
int gate_counter(cudaStream_t stream, unsigned int **out) {
    static std::mutex mu;
    static unsigned int *base[kMaxDevices] = {};
    static unsigned int next[kMaxDevices] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        set_error("lamq_xtx_accumulate: no usable current device");
        return LAMQ_ERR_CUDA;
    }
    unsigned int *slot;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (base[dev] == nullptr) {
            void *sym = nullptr;
            e = cudaGetSymbolAddress(&sym, g_gate);
            if (e != cudaSuccess || sym == nullptr) {
                set_error("lamq_xtx_accumulate: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
                return LAMQ_ERR_CUDA;
            }
            base[dev] = reinterpret_cast<unsigned int *>(sym);
        }
        slot = base[dev] + (next[dev]++ % kGateSlots);
    }
    e = cudaMemsetAsync(slot, 0, sizeof(unsigned int), stream);
    if (e != cudaSuccess) {
        set_error("lamq_xtx_accumulate: %s", cudaGetErrorString(e));
        return LAMQ_ERR_CUDA;
    }
    *out = slot;
    return LAMQ_OK;
}

// A stream-ordered memory pool of the library's own per device, keeping what it has grown to (the last-window scratch
// of a launch is allocated and freed on the launch's stream; with the default pool's release threshold of zero every
// launch would map its scratch anew).
int scratch_pool(cudaMemPool_t *out) {
    static std::mutex mu;
    static cudaMemPool_t pools[kMaxDevices] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        set_error("lamq_xtx_accumulate: no usable current device");
        return LAMQ_ERR_CUDA;
    }
    std::lock_guard<std::mutex> lock(mu);
    if (pools[dev] == nullptr) {
        cudaMemPoolProps props{};
        props.allocType = cudaMemAllocationTypePinned;
        props.location.type = cudaMemLocationTypeDevice;
        props.location.id = dev;
        cudaMemPool_t pool = nullptr;
        e = cudaMemPoolCreate(&pool, &props);
        if (e == cudaSuccess) {
            uint64_t keep = UINT64_MAX;
            e = cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
        }
        if (e != cudaSuccess) {
            set_error("lamq_xtx_accumulate: scratch pool: %s", cudaGetErrorString(e));
            return LAMQ_ERR_CUDA;
        }
        pools[dev] = pool;
    }
    *out = pools[dev];
    return LAMQ_OK;
}

int num_sms() {
    static int sms = 0;
    if (sms == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (sms <= 0) sms = 148;
    }
    return sms;
}

}  // namespace

}  // namespace lamq

using namespace lamq;

extern "C" int lamq_xtx_accumulate_scaled(const uint16_t *A, int64_t lda, const uint16_t *B, int64_t ldb,
                                          int64_t tokens, int d, int symmetric, float scale, float *acc, int64_t ldacc,
                                          int64_t chunk_tokens, int *status, lamq_stream_t stream);

extern "C" int lamq_xtx_accumulate(const uint16_t *A, int64_t lda, const uint16_t *B, int64_t ldb, int64_t tokens,
                                   int d, int symmetric, float *acc, int64_t ldacc, int64_t chunk_tokens, int *status,
                                   lamq_stream_t stream) {
    return lamq_xtx_accumulate_scaled(A, lda, B, ldb, tokens, d, symmetric, 1.0f, acc, ldacc, chunk_tokens, status,
                                      stream);
}

extern "C" int lamq_xtx_accumulate_scaled(const uint16_t *A, int64_t lda, const uint16_t *B, int64_t ldb,
                                          int64_t tokens, int d, int symmetric, float scale, float *acc, int64_t ldacc,
                                          int64_t chunk_tokens, int *status, lamq_stream_t stream) {
    LAMQ_REQUIRE(tokens >= 0 && d > 0, "lamq_xtx_accumulate: bad shape");
    if (tokens == 0) return LAMQ_OK;
    LAMQ_REQUIRE(A && B && acc && status, "lamq_xtx_accumulate: null pointer");
    LAMQ_REQUIRE(d % 8 == 0 && lda % 8 == 0 && ldb % 8 == 0 && lda >= d && ldb >= d,
                 "lamq_xtx_accumulate: d and leading dimensions must be multiples of 8 (16-byte rows for TMA)");
    LAMQ_REQUIRE(((uintptr_t)A % 16) == 0 && ((uintptr_t)B % 16) == 0, "lamq_xtx_accumulate: operands not 16-byte aligned");
    LAMQ_REQUIRE(ldacc >= d, "lamq_xtx_accumulate: accumulator leading dimension below d");
    LAMQ_REQUIRE(chunk_tokens >= BK && chunk_tokens % BK == 0, "lamq_xtx_accumulate: chunk_tokens must be a multiple of 64");
    CUtensorMap ma, mb;
    int st = make_map(&ma, A, tokens, d, lda, "lamq_xtx_accumulate");
    if (st != LAMQ_OK) return st;
    st = make_map(&mb, B, tokens, d, ldb, "lamq_xtx_accumulate");
    if (st != LAMQ_OK) return st;
    GemmParams p{};
    p.acc = acc;
    p.ldc = ldacc;
    p.d = d;
    p.scale = scale;
    // contractions of d >= 512 run on CTA pairs (256 x 256 tiles), smaller ones on single CTAs (128 x 256)
    p.pair = d >= 512 ? 1 : 0;
    const int tm = p.pair ? 256 : BM;
    p.nti = (d + tm - 1) / tm;
    p.ntj = (d + BN - 1) / BN;
    {
        const int target = p.pair ? kPairBandTarget : kBandTarget;
        const int nb = (p.nti + target - 1) / target;
        p.band = (p.nti + nb - 1) / nb;
    }
    p.kblocks = (int)((tokens + BK - 1) / BK);
    p.kblocks_per_chunk = (int)(chunk_tokens / BK);
    p.nchunk = (p.kblocks + p.kblocks_per_chunk - 1) / p.kblocks_per_chunk;
    p.symmetric = symmetric ? 1 : 0;
    p.status = status;
    int64_t tiles = 0;
    for (int ti = 0; ti < p.nti; ++ti)
        tiles += symmetric ? std::max(0, p.ntj - (p.pair ? ti : ti / 2)) : p.ntj;
    p.units = tiles * p.nchunk;
    p.ntiles = tiles;
    st = gate_counter((cudaStream_t)stream, &p.gate);
    if (st != LAMQ_OK) return st;
    // the last window (tiles beyond the last full one) goes through scratch slots when its tiles have several chunks
    const int grid_units = (int)std::min<int64_t>(p.units, p.pair ? num_sms() / 2 : num_sms());
    p.last0 = tiles / grid_units * grid_units;
    p.last_tiles = (int)(tiles - p.last0);
    float *scratch = nullptr;
    const size_t scratch_bytes = (size_t)p.nchunk * p.last_tiles * 2 * kSlotFloats * sizeof(float);
    if (p.nchunk > 1 && p.last_tiles > 0) {
        cudaMemPool_t pool = nullptr;
        st = scratch_pool(&pool);
        if (st != LAMQ_OK) return st;
        const cudaError_t ea =
            cudaMallocFromPoolAsync(reinterpret_cast<void **>(&scratch), scratch_bytes, pool, (cudaStream_t)stream);
        if (ea != cudaSuccess) {
            set_error("lamq_xtx_accumulate: %zu bytes of scratch: %s", scratch_bytes, cudaGetErrorString(ea));
            return LAMQ_ERR_CUDA;
        }
        p.scratch = scratch;
    }
    auto fail = [&](cudaError_t err) {
        set_error("lamq_xtx_accumulate: %s", cudaGetErrorString(err));
        if (scratch != nullptr) cudaFreeAsync(scratch, (cudaStream_t)stream);
        return LAMQ_ERR_CUDA;
    };
    cudaError_t e;
    if (p.pair) {
        const int64_t clusters = std::min<int64_t>(p.units, num_sms() / 2);
        p.win = (int)clusters;
        e = smem_limit_once((const void *)xtx_pair_kernel, (int)kPairSmemBytes);
        if (e != cudaSuccess) return fail(e);
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3((unsigned)(2 * clusters), 1, 1);
        cfg.blockDim = dim3(kThreads, 1, 1);
        cfg.dynamicSmemBytes = kPairSmemBytes;
        cfg.stream = (cudaStream_t)stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        e = cudaLaunchKernelEx(&cfg, xtx_pair_kernel, ma, mb, p);
        if (e != cudaSuccess) return fail(e);
        count_launch();
    } else {
        e = smem_limit_once((const void *)xtx_kernel, (int)kSmemBytes);
        if (e != cudaSuccess) return fail(e);
        const int64_t grid = p.units < num_sms() ? p.units : num_sms();
        p.win = (int)grid;
        xtx_kernel<<<(unsigned)grid, kThreads, kSmemBytes, (cudaStream_t)stream>>>(ma, mb, p);
        e = cudaGetLastError();
        if (e != cudaSuccess) return fail(e);
        count_launch();
    }
    if (scratch != nullptr) {
        last_window_reduce_kernel<<<dim3(kSlotFloats / 256 / 8, 2 * p.last_tiles), 256, 0, (cudaStream_t)stream>>>(p);
        e = cudaGetLastError();
        if (e != cudaSuccess) return fail(e);
        count_launch();
        e = cudaFreeAsync(scratch, (cudaStream_t)stream);
        if (e != cudaSuccess) {
            set_error("lamq_xtx_accumulate: %s", cudaGetErrorString(e));
            return LAMQ_ERR_CUDA;
        }
    }
    return LAMQ_OK;
}

extern "C" int lamq_weighted_split(const uint16_t *scaled, int64_t lds, const uint16_t *plain, int64_t ldp,
                                   const float *w, const int32_t *idx, int64_t nw, int d, uint16_t *out_split,
                                   uint16_t *out_plain, lamq_stream_t stream) {
    LAMQ_REQUIRE(nw >= 0 && d > 0, "lamq_weighted_split: bad shape");
    if (nw == 0) return LAMQ_OK;
    LAMQ_REQUIRE(scaled && plain && w && idx && out_split && out_plain, "lamq_weighted_split: null pointer");
    weighted_split_kernel<<<(unsigned)nw, 256, 0, (cudaStream_t)stream>>>(
        reinterpret_cast<const __nv_bfloat16 *>(scaled), lds, reinterpret_cast<const __nv_bfloat16 *>(plain), ldp, w,
        idx, nw, d, reinterpret_cast<__nv_bfloat16 *>(out_split), reinterpret_cast<__nv_bfloat16 *>(out_plain));
    LAMQ_CHECK_LAUNCH("lamq_weighted_split");
    return LAMQ_OK;
}

extern "C" int lamq_gather_rows(const uint16_t *src, int64_t lds, const int32_t *idx, int64_t n, int d, uint16_t *dst,
                                lamq_stream_t stream) {
    LAMQ_REQUIRE(n >= 0 && d > 0 && d % 8 == 0 && lds % 8 == 0 && lds >= d, "lamq_gather_rows: bad shape");
    if (n == 0) return LAMQ_OK;
    LAMQ_REQUIRE(src && idx && dst, "lamq_gather_rows: null pointer");
    LAMQ_REQUIRE(((uintptr_t)src % 16) == 0 && ((uintptr_t)dst % 16) == 0, "lamq_gather_rows: rows not 16-byte aligned");
    const int units = d / 8;
    const int64_t work = n * units;
    const int blocks = (int)std::min<int64_t>((work + 255) / 256, 148 * 16);
    gather_rows_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(reinterpret_cast<const uint4 *>(src), lds / 8, idx, n,
                                                                 units, reinterpret_cast<uint4 *>(dst));
    LAMQ_CHECK_LAUNCH("lamq_gather_rows");
    return LAMQ_OK;
}

extern "C" int lamq_hessian_finalize(const float *accH, const float *accD, int d, int64_t ld, double n_tok, double *H,
                                     double *D, lamq_stream_t stream) {
    LAMQ_REQUIRE(d > 0 && ld >= d && n_tok > 0, "lamq_hessian_finalize: bad shape");
    LAMQ_REQUIRE(accH && H && (accD == nullptr) == (D == nullptr), "lamq_hessian_finalize: null pointer");
    const int64_t n = (int64_t)d * d;
    const int blocks = (int)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
    finalize_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(accH, accD, ld, d, 1.0 / n_tok, H, D);
    LAMQ_CHECK_LAUNCH("lamq_hessian_finalize");
    return LAMQ_OK;
}
