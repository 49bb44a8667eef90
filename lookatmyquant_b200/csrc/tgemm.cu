// The trellis-dequant GEMM on tcgen05: Y = X · Wᵀ with W decoded from trellis states straight into the tensor
// cores' shared-memory operand, never written to HBM.
//
// Reference: the product of runtime_mlx/fast_q35.py:69-201 (y = S ⊙ (V[state]·(R_in x)), there as Metal kernels for
// one vector) and compiler_artifact.py:433-442 (decode_rotated: W_rj = V[state_rj]·S_r). For many input vectors the
// reference decodes W and multiplies densely; here the decode is fused into a bf16 GEMM with fp32 accumulation:
//   Y[v][map[r]] = S_r · Σ_j bf16(V[state_rj]) · X[v][j]
// for every row group of a launch (the groups of the matrices that read one input, as the grouped product takes).
// States come from the opgraph-packed-1 stream (state_j = the L bits at bit (N − 1 − j)·k of the reversed row
// stream, packed.cu) or from an int16 state matrix (a TrellisWord's states, row or column trellis).
//
// Tiles: a pair of CTAs (a cluster of two, cta_group::2 MMAs with M = 256, N = bn <= 256, K = 16) takes 256 weight
// rows: each CTA decodes its 128 rows into its own shared memory and loads its half of each block of bn input vectors
// (bn / 2 rows of X), and each CTA's TMEM holds its 128 rows x bn outputs. A work unit is (256-row tile, block of
// NACC·bn vectors); with NACC = 2 both accumulators share each decoded slice (the decode is amortised over 512
// vectors), with NACC = 1 they alternate between units so the epilogue of one unit overlaps the next one's MMAs.
// Pairing halves the X traffic from L2 per multiply-add (each X tile feeds 256 rows) and the X bytes each CTA stages,
// so the ring has 4 (or 6) stages of 64 columns. No TMA multicast: each CTA loads its own half.
//
// Warp roles (448 threads a CTA): warp 0 issues the TMA loads of X (K-major, 128-byte swizzle) in both CTAs, warp 1
// allocates the pair's TMEM and (in the even CTA, one thread) issues the MMAs, warps 2-9 decode (two threads per row,
// 32 columns of each slice each: a thread reads its part of the row's stream — two slices ahead — cuts the states
// out with funnel shifts, looks them up in the CTA's bf16 copy of the table and stores them as four 16-byte chunks in
// the 128-byte-swizzled K-major layout the MMA descriptor reads, then its warp arrives on the even CTA's stage
// barrier), warps 10-13 drain the accumulators (row scale, optional map, fp32 or bf16 out). The even CTA's MMA
// commits release both CTAs' stages and accumulators (multicast commit); both CTAs' drain threads release an
// accumulator on the even CTA's barrier. Every wait is bounded (2 s): a timeout sets the status word and the pair
// winds down.
#include <algorithm>
#include <climits>
#include <utility>
#include <vector>

#include <cuda.h>
#include <cuda_bf16.h>

#include "lamq_common.cuh"
#include "sm100.cuh"

namespace lamq {
namespace {

using namespace sm100;

constexpr int TM = 128, TN = 256, TK = 64;     // rows a CTA decodes, vectors an accumulator holds, K per slice
constexpr int TM2 = 2 * TM;                     // rows of a pair's tile
constexpr int A_BYTES = TM * TK * 2, B_BYTES = (TN / 2) * TK * 2;  // a CTA's A slice, its half of an X block
constexpr int kDecWarps = 8, kEpiWarps = 4;
constexpr int kParts = kDecWarps / 4;      // decoder threads per row: each takes 64 / kParts columns of a slice
constexpr int kCols = TK / kParts;         // columns of a slice per decoder thread
constexpr int kDecBar = 1;                 // named barrier of the decoder warps (table reloads)
constexpr int kThreads = (2 + kDecWarps + kEpiWarps) * 32;
constexpr uint32_t kTmemCols = 512;
constexpr int kTableEntries = 4096;
constexpr int kMaxGemmGroups = 16;
constexpr int kMaxInputs = 4;              // distinct inputs X (tensor maps) a launch reads

struct GemmGroup {
    const uint32_t *codes;   // packed rows (rows x wpr words), or null with states
    const int16_t *states;   // int16 states (rows x lds), or null with codes
    int64_t lds;
    int64_t rows;
    int k, L;
    const float *scales;     // fp32, one per row
    const float *table;      // fp32, 2^L entries
    const uint32_t *map;     // output row of each row, or null
    void *y;                 // fp32 or bf16, nvec x ldy
    int64_t ldy;
    int input;               // which of the launch's inputs X the group multiplies
    int64_t arow;            // decode-once mode: the group's first row in its input's decoded weights
    int64_t tiles;           // 256-row tiles of the group
    int64_t first;           // the group's first unit in the launch's numbering
};

struct GemmParams {
    GemmGroup g[kMaxGemmGroups];
    int ng;
    int n[kMaxInputs], kslices[kMaxInputs];  // per input: columns and 64-column slices
    int bn;                  // vectors per accumulator (<= 256, a multiple of 16)
    int64_t nvec;
    int64_t vblocks, units;  // vector blocks of NACC·bn; units = Σ tiles x vblocks
    int y_bf16;
    int *status;
};

template <int NACC>
struct Layout {
    static constexpr int STAGES = NACC == 2 ? 4 : 6;
    static constexpr int STAGE_BYTES = A_BYTES + NACC * B_BYTES;
    static constexpr int TABLE_OFF = STAGES * STAGE_BYTES;
    static constexpr int BAR_OFF = TABLE_OFF + kTableEntries * 2;
    static constexpr size_t SMEM = 1024 + BAR_OFF + 8 * (2 * STAGES + 5) + 16;
};
static_assert(Layout<1>::SMEM <= 232448 && Layout<2>::SMEM <= 232448, "shared memory above the opt-in limit");

__device__ __forceinline__ void fence_async_shared() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void sts128(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

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

// Unit u: group g (units numbered group by group, the groups of the longest rows first, so the longest units are
// handed out first), then its 256-row tile and vector block (consecutive units share the tile).
__device__ __forceinline__ void unit_of(const GemmParams &p, int64_t u, int &vb, int &g, int64_t &rt) {
    g = 0;
    while (g + 1 < p.ng && p.g[g + 1].first <= u) ++g;
    const int64_t local = u - p.g[g].first;
    rt = local / p.vblocks;
    vb = (int)(local % p.vblocks);
}

// Stream words of one decoder thread's part of a slice: columns c0 + part·kCols + i' (i' < kCols) sit at stream bit
// offsets (kCols − 1 − i')·K above the part's word-aligned base (N − c0 − 64)·K + (kParts − 1 − part)·kCols·K.
template <int K>
struct Slice {
    static constexpr int NW = ((kCols - 1) * K + 12 + 31) / 32;
    uint32_t w[NW];
};

template <int K>
__device__ __forceinline__ void load_slice(Slice<K> &s, const uint32_t *row, int wpr, int N, int c0, int part,
                                           bool live) {
    const int wb = (((N - c0 - 64) * K) >> 5) + (kParts - 1 - part) * kCols * K / 32;  // may be negative
#pragma unroll
    for (int q = 0; q < Slice<K>::NW; ++q) {
        const int w = wb + q;
        s.w[q] = (live && w >= 0 && w < wpr) ? __ldg(row + w) : 0u;
    }
}

__device__ __forceinline__ uint32_t bf16_pair(const uint16_t *tab, uint32_t s0, uint32_t s1) {
    return (uint32_t)tab[s0] | ((uint32_t)tab[s1] << 16);
}

// Decodes the thread's kCols states of a slice and stores them as bf16 (kCols / 8 chunks of 16 bytes, swizzled).
// `valid`: columns of the part below n (the rest are written as zeros).
template <int K>
__device__ __forceinline__ void store_slice_packed(const Slice<K> &s, const uint16_t *tab, uint32_t lmask,
                                                   uint32_t arow, int cbase, int swz, int valid) {
#pragma unroll
    for (int c = 0; c < kCols / 8; ++c) {
        uint32_t pk[4];
#pragma unroll
        for (int h = 0; h < 4; ++h) {
            uint32_t st[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int i = 8 * c + 2 * h + e;
                const int o = (kCols - 1 - i) * K;
                st[e] = __funnelshift_r(s.w[o >> 5], s.w[(o >> 5) + 1], o & 31) & lmask;
            }
            pk[h] = bf16_pair(tab, st[0], st[1]);
            if (8 * c + 2 * h >= valid) pk[h] = 0u;
            else if (8 * c + 2 * h + 1 >= valid) pk[h] &= 0xFFFFu;
        }
        sts128(arow + ((uint32_t)((cbase + c) ^ swz) << 4), pk[0], pk[1], pk[2], pk[3]);
    }
}

__device__ __forceinline__ void store_slice_states(const uint4 (&v)[kCols / 8], const uint16_t *tab, uint32_t lmask,
                                                   uint32_t arow, int cbase, int swz, int valid) {
#pragma unroll
    for (int c = 0; c < kCols / 8; ++c) {
        const uint32_t raw[4] = {v[c].x, v[c].y, v[c].z, v[c].w};
        uint32_t pk[4];
#pragma unroll
        for (int h = 0; h < 4; ++h) {
            pk[h] = bf16_pair(tab, raw[h] & lmask, (raw[h] >> 16) & lmask);
            if (8 * c + 2 * h >= valid) pk[h] = 0u;
            else if (8 * c + 2 * h + 1 >= valid) pk[h] &= 0xFFFFu;
        }
        sts128(arow + ((uint32_t)((cbase + c) ^ swz) << 4), pk[0], pk[1], pk[2], pk[3]);
    }
}

__device__ __forceinline__ void load_states(uint4 (&v)[kCols / 8], const int16_t *row, int c0, int n, bool live) {
#pragma unroll
    for (int c = 0; c < kCols / 8; ++c) {
        const int j = c0 + 8 * c;
        v[c] = (live && j < n) ? __ldg(reinterpret_cast<const uint4 *>(row + j)) : make_uint4(0, 0, 0, 0);
    }
}

// The decode of one unit's slices by decoder thread d: row d % 128 of the tile, columns part·kCols.. of each slice
// (part = d / 128). The next two slices' codes are in flight while one is decoded. With ok false (a wait gave up
// earlier) the thread only walks the unit, so every decoder meets the same named barriers.
template <int K, int NACC>
__device__ void decode_unit(const GemmParams &p, const GemmGroup &g, int64_t rt, int d, const uint16_t *tab,
                            uint32_t smem_base, uint32_t full0, uint32_t empty0, int &stage, uint32_t &phase,
                            bool &ok, uint32_t rank) {
    using LY = Layout<NACC>;
    const int r = d % TM, part = d / TM;
    const int64_t row = rt * TM2 + rank * TM + r;
    const bool live = row < g.rows;
    const uint32_t lmask = (1u << g.L) - 1u;
    const int swz = r & 7, cbase = part * (kCols / 8);
    const int lane = threadIdx.x & 31;
    const int n = p.n[g.input], kslices = p.kslices[g.input];
    const int col0 = part * kCols;
    auto publish = [&](auto &&store) {
        if (ok && !mbar_wait(empty0 + 8 * stage, phase ^ 1, p.status)) ok = false;
        if (ok) {
            store(smem_base + stage * LY::STAGE_BYTES + r * 128);
            fence_async_shared();
            __syncwarp();
            if (lane == 0) {  // the even CTA's barrier counts both CTAs' decoder warps
                if (rank == 0) mbar_arrive(full0 + 8 * stage);
                else mbar_arrive_cluster(map_to_rank(full0 + 8 * stage, 0));
            }
        }
        if (++stage == LY::STAGES) {
            stage = 0;
            phase ^= 1;
        }
    };
    if constexpr (K == 0) {
        const int16_t *srow = g.states + (live ? row : 0) * g.lds;
        uint4 cur[kCols / 8], nx1[kCols / 8], nx2[kCols / 8];
        load_states(cur, srow, col0, n, live && ok);
        load_states(nx1, srow, TK + col0, n, live && ok && kslices > 1);
        for (int kb = 0; kb < kslices; ++kb) {
            load_states(nx2, srow, (kb + 2) * TK + col0, n, live && ok && kb + 2 < kslices);
            const int valid = live ? n - kb * TK - col0 : 0;
            publish([&](uint32_t arow) { store_slice_states(cur, tab, lmask, arow, cbase, swz, valid); });
#pragma unroll
            for (int c = 0; c < kCols / 8; ++c) {
                cur[c] = nx1[c];
                nx1[c] = nx2[c];
            }
        }
    } else {
        const int N = (n + 31) / 32 * 32;
        const int wpr = N / 32 * K;
        const uint32_t *crow = g.codes + (live ? row : 0) * (int64_t)wpr;
        Slice<K> cur, nx1, nx2;
        load_slice<K>(cur, crow, wpr, N, 0, part, live && ok);
        load_slice<K>(nx1, crow, wpr, N, TK, part, live && ok && kslices > 1);
        for (int kb = 0; kb < kslices; ++kb) {
            load_slice<K>(nx2, crow, wpr, N, (kb + 2) * TK, part, live && ok && kb + 2 < kslices);
            const int valid = live ? n - kb * TK - col0 : 0;
            publish([&](uint32_t arow) { store_slice_packed<K>(cur, tab, lmask, arow, cbase, swz, valid); });
            cur = nx1;
            nx1 = nx2;
        }
    }
}

template <int NACC, bool ATMA>
__global__ void __launch_bounds__(kThreads, 1)
    trellis_gemm_kernel(const __grid_constant__ CUtensorMap map0, const __grid_constant__ CUtensorMap map1,
                        const __grid_constant__ CUtensorMap map2, const __grid_constant__ CUtensorMap map3,
                        const __grid_constant__ CUtensorMap amap0, const __grid_constant__ CUtensorMap amap1,
                        const __grid_constant__ CUtensorMap amap2, const __grid_constant__ CUtensorMap amap3,
                        const __grid_constant__ GemmParams p) {
    using LY = Layout<NACC>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + LY::BAR_OFF);
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 2 * LY::STAGES + 5);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const bool leader = rank == 0;
    const int64_t cluster = blockIdx.x >> 1, nclusters = gridDim.x >> 1;
    const uint32_t smem_base = smem_u32(smem);
    const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + LY::STAGES);
    const uint32_t tfull0 = smem_u32(bars + 2 * LY::STAGES), tempty0 = smem_u32(bars + 2 * LY::STAGES + 2);
    const uint32_t drain = smem_u32(bars + 2 * LY::STAGES + 4);
    if (threadIdx.x == 0) {
        for (int s = 0; s < LY::STAGES; ++s) {
            // used on the even CTA: its expect_tx (both CTAs' bytes) + one arrival per decoder warp of both CTAs
            // (decode-once mode: the weights arrive by TMA too, and the expect_tx is the only arrival)
            mbar_init(full0 + 8 * s, ATMA ? 1 : 1 + 2 * kDecWarps);
            mbar_init(empty0 + 8 * s, 1);  // the even CTA's multicast commit
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(tfull0 + 8 * a, 1);
            mbar_init(tempty0 + 8 * a, 2 * kEpiWarps * 32);  // both CTAs' drain threads (used on the even CTA)
        }
        mbar_init(drain, 1);
        fence_mbar_init();
        prefetch_tmap(&map0);
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
    const int bn = p.bn, hb = bn / 2;  // vectors an accumulator holds; a CTA's half of them
    const uint32_t half_tx = (uint32_t)hb * TK * 2;

    if (warp == 0) {
        if (lane == 0) {  // ---- TMA producer (both CTAs: each loads its half of each X block)
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int64_t u = cluster; ok && u < p.units; u += nclusters) {
                int vb, g;
                int64_t rt;
                unit_of(p, u, vb, g, rt);
                const int in = p.g[g].input;
                const CUtensorMap *mapX = in == 0 ? &map0 : in == 1 ? &map1 : in == 2 ? &map2 : &map3;
                const CUtensorMap *mapA = in == 0 ? &amap0 : in == 1 ? &amap1 : in == 2 ? &amap2 : &amap3;
                const int arow = (int)(p.g[g].arow + rt * TM2 + rank * TM);
                for (int kb = 0; kb < p.kslices[in]; ++kb) {
                    if (!mbar_wait(empty0 + 8 * stage, phase ^ 1, p.status)) {
                        ok = false;
                        break;
                    }
                    if (leader) mbar_expect_tx(full0 + 8 * stage, 2 * (NACC * half_tx + (ATMA ? A_BYTES : 0)));
                    const uint32_t fb = map_to_rank(full0 + 8 * stage, 0);
                    const uint32_t sb = smem_base + stage * LY::STAGE_BYTES + A_BYTES;
                    if (ATMA) tma_load_2d_pair(sb - A_BYTES, mapA, kb * TK, arow, fb);
#pragma unroll
                    for (int j = 0; j < NACC; ++j)
                        tma_load_2d_pair(sb + j * B_BYTES, mapX, kb * TK, (vb * NACC + j) * bn + (int)rank * hb, fb);
                    if (++stage == LY::STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            if (!ok) __nanosleep(200000);  // error path: the copies in flight land (their barrier is the even CTA's)
        }
    } else if (warp == 1) {
        if (lane == 0 && leader) {  // ---- MMA issuer (the even CTA)
            const uint32_t idesc = idesc_bf16_f32(TM2, bn, false, false);
            int stage = 0;
            uint32_t phase = 0;
            uint32_t uses[2] = {0, 0};
            int64_t it = 0;
            bool ok = true;
            for (int64_t u = cluster; ok && u < p.units; u += nclusters, ++it) {
                int vb_, g_;
                int64_t rt_;
                unit_of(p, u, vb_, g_, rt_);
                const int kslices = p.kslices[p.g[g_].input];
                int slot[NACC];
#pragma unroll
                for (int j = 0; j < NACC; ++j) {
                    slot[j] = NACC == 2 ? j : (int)(it & 1);
                    if (ok && !mbar_wait_cluster(tempty0 + 8 * slot[j], (uses[slot[j]] & 1) ^ 1, p.status)) ok = false;
                    ++uses[slot[j]];
                }
                if (!ok) break;
                tc_fence_after();
                for (int kb = 0; kb < kslices; ++kb) {
                    if (!mbar_wait_cluster(full0 + 8 * stage, phase, p.status)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = smem_base + stage * LY::STAGE_BYTES, sb = sa + A_BYTES;
                    // the two accumulators' MMAs alternate per 16 columns: consecutive MMAs read the same A sub-tile
#pragma unroll
                    for (int kk = 0; kk < TK / 16; ++kk) {
                        const uint64_t ad = smem_desc_sw128(sa + kk * 32, 16, 1024);
#pragma unroll
                        for (int j = 0; j < NACC; ++j) {
                            const uint64_t bd = smem_desc_sw128(sb + j * B_BYTES + kk * 32, 16, 1024);
                            mma_f16_ss_pair(tmem + slot[j] * TN, ad, bd, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
                        }
                    }
                    mma_commit_pair_multicast(empty0 + 8 * stage, 0x3);
                    if (++stage == LY::STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (!ok) break;
#pragma unroll
                for (int j = 0; j < NACC; ++j) mma_commit_pair_multicast(tfull0 + 8 * slot[j], 0x3);
            }
            // every MMA this thread issued completes before TMEM is released
            mma_commit_pair(drain);
            const unsigned long long t0 = globaltimer();
            while (!mbar_try_wait(drain, 0) && globaltimer() - t0 < kWaitTimeoutNs) {
            }
        }
    } else if (warp < 2 + kDecWarps) {  // ---- decoders: thread d owns part d / 128 of row d % 128 of its half
      if (!ATMA) {  // (decode-once mode: the weights were decoded before the launch)
        const int d = threadIdx.x - 64;
        uint16_t *tab = reinterpret_cast<uint16_t *>(smem + LY::TABLE_OFF);
        int stage = 0;
        uint32_t phase = 0;
        int cur_group = -1;
        bool ok = true;
        for (int64_t u = cluster; u < p.units; u += nclusters) {
            int vb, gi;
            int64_t rt;
            unit_of(p, u, vb, gi, rt);
            const GemmGroup &g = p.g[gi];
            if (gi != cur_group) {  // the group's table as bf16 (every decoder takes this branch together)
                asm volatile("bar.sync %0, %1;" ::"r"(kDecBar), "r"(kDecWarps * 32) : "memory");
                const int nt = 1 << g.L;
                for (int i = d; i < kTableEntries; i += kDecWarps * 32) {
                    const float v = i < nt ? __ldg(g.table + i) : 0.f;
                    tab[i] = __bfloat16_as_ushort(__float2bfloat16_rn(v));
                }
                asm volatile("bar.sync %0, %1;" ::"r"(kDecBar), "r"(kDecWarps * 32) : "memory");
                cur_group = gi;
            }
            switch (g.states ? 0 : g.k) {
                case 0: decode_unit<0, NACC>(p, g, rt, d, tab, smem_base, full0, empty0, stage, phase, ok, rank); break;
                case 1: decode_unit<1, NACC>(p, g, rt, d, tab, smem_base, full0, empty0, stage, phase, ok, rank); break;
                case 2: decode_unit<2, NACC>(p, g, rt, d, tab, smem_base, full0, empty0, stage, phase, ok, rank); break;
                case 3: decode_unit<3, NACC>(p, g, rt, d, tab, smem_base, full0, empty0, stage, phase, ok, rank); break;
                default: decode_unit<4, NACC>(p, g, rt, d, tab, smem_base, full0, empty0, stage, phase, ok, rank); break;
            }
        }
      }
    } else {  // ---- epilogue (both CTAs): warp w reads TMEM lanes 32·(w % 4).. (rows of this CTA's half)
        const int q = warp & 3;
        const bool remote = !leader;  // the odd CTA's threads arrive on the even CTA's barrier
        uint32_t uses[2] = {0, 0};
        int64_t it = 0;
        bool ok = true;
        for (int64_t u = cluster; ok && u < p.units; u += nclusters, ++it) {
            int vb, gi;
            int64_t rt;
            unit_of(p, u, vb, gi, rt);
            const GemmGroup &g = p.g[gi];
            const int64_t row = rt * TM2 + rank * TM + 32 * q + lane;
            const bool live = row < g.rows;
            const float scale = live ? __ldg(g.scales + row) : 0.f;
            const int64_t orow = live ? (g.map ? (int64_t)__ldg(g.map + row) : row) : 0;
#pragma unroll 1
            for (int j = 0; j < NACC; ++j) {
                const int slot = NACC == 2 ? j : (int)(it & 1);
                if (!mbar_wait(tfull0 + 8 * slot, uses[slot] & 1, p.status)) {
                    ok = false;
                    break;
                }
                ++uses[slot];
                tc_fence_after();
                const int64_t v0 = (int64_t)(vb * NACC + j) * bn;
#pragma unroll 1
                for (int c = 0; c < bn / 32; ++c) {
                    uint32_t r[32];
                    tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + slot * TN + c * 32, r);
                    tmem_ld_wait();
                    if (live) {
                        const int64_t vc = v0 + c * 32;
                        if (p.y_bf16) {
                            uint16_t *y = reinterpret_cast<uint16_t *>(g.y) + orow;
#pragma unroll
                            for (int e = 0; e < 32; ++e)
                                if (vc + e < p.nvec)
                                    y[(vc + e) * g.ldy] =
                                        __bfloat16_as_ushort(__float2bfloat16_rn(__uint_as_float(r[e]) * scale));
                        } else {
                            float *y = reinterpret_cast<float *>(g.y) + orow;
#pragma unroll
                            for (int e = 0; e < 32; ++e)
                                if (vc + e < p.nvec) y[(vc + e) * g.ldy] = __uint_as_float(r[e]) * scale;
                        }
                    }
                }
                if (bn % 32) {  // a last chunk of 16 columns
                    const int c0 = bn / 32 * 32;
                    uint32_t r[16];
                    tmem_ld16(tmem + ((uint32_t)(32 * q) << 16) + slot * TN + c0, r);
                    tmem_ld_wait();
                    if (live) {
                        const int64_t vc = v0 + c0;
#pragma unroll
                        for (int e = 0; e < 16; ++e) {
                            if (vc + e >= p.nvec) continue;
                            const float val = __uint_as_float(r[e]) * scale;
                            if (p.y_bf16)
                                reinterpret_cast<uint16_t *>(g.y)[(vc + e) * g.ldy + orow] =
                                    __bfloat16_as_ushort(__float2bfloat16_rn(val));
                            else
                                reinterpret_cast<float *>(g.y)[(vc + e) * g.ldy + orow] = val;
                        }
                    }
                }
                tc_fence_before();
                if (remote) mbar_arrive_cluster(map_to_rank(tempty0 + 8 * slot, 0));
                else mbar_arrive(tempty0 + 8 * slot);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync_all();  // neither CTA leaves while the pair's MMAs or arrivals may still touch it
    tc_fence_after();
    if (warp == 1) tmem_dealloc_pair(tmem, kTmemCols);
}

// ---- decode-once mode: the groups' weights decoded to bf16 rows before the GEMM, which then loads them by TMA

struct DecodeGroup {
    const uint32_t *codes;
    const int16_t *states;
    int64_t lds, rows;
    int k, L, n;
    const float *table;
    uint16_t *out;           // rows x ld bf16
    int64_t ld;
    int64_t first_block;     // the group's first block of the decode launch
};

struct DecodeParams {
    DecodeGroup g[kMaxGemmGroups];
    int ng;
};

constexpr int kDecodeThreads = 256;
constexpr int kDecodeBlocksPerSm = 8;  // resident decode blocks per SM (8 KB of table each): the grid is one wave

// The rows of one decode group from this block's share of its 8-column chunks (K = 0: int16 states; else packed
// k-bit symbols, the per-column bit offsets constants).
template <int K>
__device__ __forceinline__ void decode_items(const DecodeGroup &g, const uint16_t *tab, int64_t first, int64_t step) {
    const int nch = (int)(g.ld / 8);
    const int64_t items = g.rows * nch;
    const uint32_t lmask = (1u << g.L) - 1u;
    const int N = (g.n + 31) / 32 * 32;
    const int wpr = N / 32 * (K > 0 ? K : 1);
#pragma unroll 2
    for (int64_t it = first; it < items; it += step) {
        const int64_t r = it / nch;
        const int j0 = (int)(it % nch) * 8;
        uint32_t st[8];
        if constexpr (K == 0) {
            const uint4 v = j0 < g.n ? __ldg(reinterpret_cast<const uint4 *>(g.states + r * g.lds + j0))
                                     : make_uint4(0, 0, 0, 0);
            const uint32_t raw[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int h = 0; h < 4; ++h) {
                st[2 * h] = raw[h] & lmask;
                st[2 * h + 1] = (raw[h] >> 16) & lmask;
            }
        } else {
            // state of column j0 + i: the L bits at (N − 1 − j0 − i)·K = b0 + (7 − i)·K, b0 = (N − 8 − j0)·K; with
            // j0 a multiple of 8, b0 mod 32 is one of 32 / gcd(32, 8K) values and the 8 states span < 3 words
            const uint32_t *row = g.codes + r * (int64_t)wpr;
            const int64_t b0 = (int64_t)(N - 8 - j0) * K;
            const int w0 = (int)(b0 >> 5), sh = (int)(b0 & 31);
            uint32_t w[3];
#pragma unroll
            for (int q = 0; q < 3; ++q) w[q] = (w0 + q >= 0 && w0 + q < wpr) ? __ldg(row + w0 + q) : 0u;
            const uint64_t lo = (uint64_t)w[1] << 32 | w[0];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int off = (7 - i) * K;  // a constant
                if (7 * K + 12 <= 32) {       // all eight states inside the first 64 bits whatever sh is
                    st[i] = (uint32_t)(lo >> (sh + off)) & lmask;
                } else {
                    const int pos = sh + off;
                    st[i] = (pos < 32 ? __funnelshift_r(w[0], w[1], pos) : __funnelshift_r(w[1], w[2], pos - 32)) &
                            lmask;
                }
            }
        }
        uint32_t pk[4];
#pragma unroll
        for (int h = 0; h < 4; ++h) {
            const uint32_t a = j0 + 2 * h < g.n ? tab[st[2 * h]] : 0u;
            const uint32_t b = j0 + 2 * h + 1 < g.n ? tab[st[2 * h + 1]] : 0u;
            pk[h] = a | (b << 16);
        }
        *reinterpret_cast<uint4 *>(g.out + r * g.ld + j0) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    }
}

// bf16(table[state]) for every (row, column) of every group: a thread per 8 consecutive columns of a row (one
// 16-byte store), the states cut from three stream words (or read as eight int16), the group's table in shared
// memory as bf16. Columns from n to the row's end (ld) are written as zeros.
__global__ void __launch_bounds__(kDecodeThreads) decode_rows_kernel(const __grid_constant__ DecodeParams p) {
    __shared__ uint16_t tab[kTableEntries];
    int gi = 0;
    while (gi + 1 < p.ng && p.g[gi + 1].first_block <= blockIdx.x) ++gi;
    const DecodeGroup &g = p.g[gi];
    const int nt = 1 << g.L;
    for (int i = threadIdx.x; i < kTableEntries; i += kDecodeThreads)
        tab[i] = __bfloat16_as_ushort(__float2bfloat16_rn(i < nt ? __ldg(g.table + i) : 0.f));
    __syncthreads();
    const int64_t nblocks = (gi + 1 < p.ng ? p.g[gi + 1].first_block : gridDim.x) - g.first_block;
    const int64_t first = (blockIdx.x - g.first_block) * kDecodeThreads + threadIdx.x;
    const int64_t step = nblocks * kDecodeThreads;
    switch (g.states ? 0 : g.k) {
        case 0: decode_items<0>(g, tab, first, step); break;
        case 1: decode_items<1>(g, tab, first, step); break;
        case 2: decode_items<2>(g, tab, first, step); break;
        case 3: decode_items<3>(g, tab, first, step); break;
        default: decode_items<4>(g, tab, first, step); break;
    }
}

using EncodeTiled = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                 const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encode_fn() {
    static EncodeTiled fn = [] {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            return reinterpret_cast<EncodeTiled>(ptr);
        return static_cast<EncodeTiled>(nullptr);
    }();
    return fn;
}

int num_sms() {
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms > 0 ? sms : 148;
}

template <int NACC, bool ATMA>
int launch_gemm(const CUtensorMap *maps, const CUtensorMap *amaps, const GemmParams &p, cudaStream_t s) {
    const cudaError_t e = smem_limit_once((const void *)trellis_gemm_kernel<NACC, ATMA>, (int)Layout<NACC>::SMEM);
    if (e != cudaSuccess) {
        set_error("lamq_trellis_gemm: %s", cudaGetErrorString(e));
        return LAMQ_ERR_CUDA;
    }
    const int64_t clusters = std::min<int64_t>(p.units, num_sms() / 2);
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)(2 * clusters), 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = Layout<NACC>::SMEM;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t le = cudaLaunchKernelEx(&cfg, trellis_gemm_kernel<NACC, ATMA>, maps[0], maps[1], maps[2],
                                              maps[3], amaps[0], amaps[1], amaps[2], amaps[3], p);
    if (le != cudaSuccess) {
        set_error("lamq_trellis_gemm: %s", cudaGetErrorString(le));
        return LAMQ_ERR_CUDA;
    }
    count_launch();
    return LAMQ_OK;
}

// bf16 rows x n (leading dimension ld elements) K-major, boxes of 64 columns x box_rows rows, 128-byte swizzle.
int kmajor_map(CUtensorMap *m, const void *base, int64_t rows, int n, int64_t ld, int box_rows) {
    EncodeTiled enc = encode_fn();
    if (enc == nullptr) {
        set_error("lamq_trellis_gemm: cuTensorMapEncodeTiled is unavailable");
        return LAMQ_ERR_CUDA;
    }
    cuuint64_t dims[2] = {(cuuint64_t)n, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    cuuint32_t box[2] = {(cuuint32_t)TK, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("lamq_trellis_gemm: cuTensorMapEncodeTiled failed (%d)", (int)r);
        return LAMQ_ERR_INVALID;
    }
    return LAMQ_OK;
}

// From this many vectors on, the weights are decoded once into the workspace and loaded by TMA: the fused decode
// would repeat for every block of 512 vectors, and its table lookups (random shared-memory reads) bound the kernel.
constexpr int64_t kDecodeOnceVectors = 2 * TN + 1;

int64_t decoded_ld(int n) { return (n + 7) / 8 * 8; }  // 16-byte rows for TMA

// One launch over up to kMaxGemmGroups groups reading up to kMaxInputs inputs (groups already sorted by n, longest
// first). In decode-once mode `scratch` receives the groups' decoded rows first (input by input, groups in order).
int run_gemm(const lamq_gemm_group *const *groups, int ngroups, int64_t nvec, int y_bf16, uint16_t *scratch,
             int *status, cudaStream_t s) {
    const bool once = nvec >= kDecodeOnceVectors;
    const int nacc = once ? 1 : (nvec > TN ? 2 : 1);
    const int bn = nvec >= TN ? TN : (int)std::max<int64_t>(32, (nvec + 15) / 16 * 16);  // M = 256 takes N >= 32
    GemmParams p{};
    CUtensorMap maps[kMaxInputs], amaps[kMaxInputs];
    const void *xs[kMaxInputs] = {};
    int ninputs = 0;
    p.bn = bn;
    p.nvec = nvec;
    p.y_bf16 = y_bf16;
    p.status = status;
    p.vblocks = (nvec + (int64_t)nacc * bn - 1) / ((int64_t)nacc * bn);
    int64_t units = 0;
    int ng = 0;
    int64_t in_rows[kMaxInputs] = {};
    for (int i = 0; i < ngroups; ++i) {
        const lamq_gemm_group &g = *groups[i];
        if (g.rows == 0) continue;
        int in = 0;
        while (in < ninputs && !(xs[in] == g.x && p.n[in] == g.n)) ++in;
        if (in == ninputs) {  // a new input: its tensor map (K-major, 128-byte swizzle, half a vector block a box)
            xs[in] = g.x;
            p.n[in] = g.n;
            p.kslices[in] = (g.n + TK - 1) / TK;
            const int st = kmajor_map(&maps[in], g.x, nvec, g.n, g.ldx, bn / 2);  // each CTA loads half a block
            if (st) return st;
            ++ninputs;
        }
        GemmGroup &d = p.g[ng++];
        d.codes = g.codes;
        d.states = g.states;
        d.lds = g.lds;
        d.rows = g.rows;
        d.k = g.k;
        d.L = g.L;
        d.scales = g.scales;
        d.table = g.table;
        d.map = g.map;
        d.y = g.y;
        d.ldy = g.ldy;
        d.input = in;
        d.arow = in_rows[in];
        in_rows[in] += g.rows;
        d.tiles = (g.rows + TM2 - 1) / TM2;
        d.first = units;
        units += d.tiles * p.vblocks;
    }
    if (ng == 0) return LAMQ_OK;
    p.ng = ng;
    p.units = units;
    if (once) {
        // the scratch holds each input's groups' rows back to back (row ld = decoded_ld(n)), inputs in order
        int64_t base[kMaxInputs];
        int64_t off = 0;
        for (int in = 0; in < ninputs; ++in) {
            base[in] = off;
            off += in_rows[in] * decoded_ld(p.n[in]);
            const int st = kmajor_map(&amaps[in], scratch + base[in], in_rows[in], p.n[in], decoded_ld(p.n[in]), TM);
            if (st) return st;
        }
        DecodeParams dp{};
        int64_t total = 0;
        for (int i = 0; i < ng; ++i) total += p.g[i].rows * (decoded_ld(p.n[p.g[i].input]) / 8);
        const int64_t budget = (int64_t)num_sms() * kDecodeBlocksPerSm;
        int64_t blocks = 0;
        for (int i = 0; i < ng; ++i) {
            const GemmGroup &g = p.g[i];
            DecodeGroup &d = dp.g[i];
            const int n = p.n[g.input];
            d.codes = g.codes;
            d.states = g.states;
            d.lds = g.lds;
            d.rows = g.rows;
            d.k = g.k;
            d.L = g.L;
            d.n = n;
            d.table = g.table;
            d.ld = decoded_ld(n);
            d.out = scratch + base[g.input] + g.arow * d.ld;
            d.first_block = blocks;
            const int64_t items = g.rows * (d.ld / 8);  // one wave of blocks, split by each group's share of chunks
            blocks += std::max<int64_t>(1, std::min<int64_t>((items + kDecodeThreads - 1) / kDecodeThreads,
                                                             budget * items / std::max<int64_t>(total, 1)));
        }
        dp.ng = ng;
        LAMQ_REQUIRE(blocks <= INT_MAX, "lamq_trellis_gemm: decode grid too large");
        decode_rows_kernel<<<(unsigned)blocks, kDecodeThreads, 0, s>>>(dp);
        LAMQ_CHECK_LAUNCH("lamq_trellis_gemm decode");
    }
    for (int in = ninputs; in < kMaxInputs; ++in) maps[in] = maps[0];
    if (!once)
        for (int in = 0; in < kMaxInputs; ++in) amaps[in] = maps[0];
    else
        for (int in = ninputs; in < kMaxInputs; ++in) amaps[in] = amaps[0];
    if (once) return launch_gemm<1, true>(maps, amaps, p, s);
    return nacc == 2 ? launch_gemm<2, false>(maps, amaps, p, s) : launch_gemm<1, false>(maps, amaps, p, s);
}

int check_groups(const lamq_gemm_group *groups, int ngroups, int64_t nvec, std::vector<const lamq_gemm_group *> &order) {
    for (int i = 0; i < ngroups; ++i) {
        const lamq_gemm_group &g = groups[i];
        LAMQ_REQUIRE(g.rows >= 0, "lamq_trellis_gemm: group %d has %lld rows", i, (long long)g.rows);
        if (g.rows == 0) continue;
        LAMQ_REQUIRE(g.n > 0 && g.ldx >= g.n, "lamq_trellis_gemm: group %d: bad input shape (n %d, ldx %lld)", i, g.n,
                     (long long)g.ldx);
        LAMQ_REQUIRE(g.rows <= INT_MAX / 2, "lamq_trellis_gemm: group %d: too many rows", i);
        LAMQ_REQUIRE(g.scales && g.table && g.y && g.x, "lamq_trellis_gemm: group %d: null pointer", i);
        LAMQ_REQUIRE(g.ldx % 8 == 0 && ((uintptr_t)g.x % 16) == 0,
                     "lamq_trellis_gemm: group %d: x must be 16-byte aligned with a leading dimension that is a "
                     "multiple of 8", i);
        LAMQ_REQUIRE((g.codes != nullptr) != (g.states != nullptr),
                     "lamq_trellis_gemm: group %d: give packed codes or int16 states, not both", i);
        LAMQ_REQUIRE(g.L >= 1 && g.L <= 12, "lamq_trellis_gemm: group %d: L in 1..12 (got %d)", i, g.L);
        if (g.codes) {
            LAMQ_REQUIRE(g.k >= 1 && g.k <= 4 && g.L > g.k,
                         "lamq_trellis_gemm: group %d: packed widths k in 1..4 and L in k+1..12 (k %d, L %d)", i, g.k,
                         g.L);
        } else {
            LAMQ_REQUIRE(g.n % 8 == 0 && g.lds >= g.n && g.lds % 8 == 0 && ((uintptr_t)g.states % 16) == 0,
                         "lamq_trellis_gemm: group %d: int16 states need n and lds multiples of 8 and 16-byte rows", i);
        }
        LAMQ_REQUIRE(nvec <= 1 || g.ldy >= g.rows, "lamq_trellis_gemm: group %d: ldy %lld below its %lld rows", i,
                     (long long)g.ldy, (long long)g.rows);
        order.push_back(&g);
    }
    // the longest rows first (their units are handed out first), stable
    std::stable_sort(order.begin(), order.end(),
                     [](const lamq_gemm_group *a, const lamq_gemm_group *b) { return a->n > b->n; });
    return LAMQ_OK;
}

// Launch batches: at most kMaxGemmGroups groups and kMaxInputs inputs each, in order.
std::vector<std::pair<size_t, size_t>> batches(const std::vector<const lamq_gemm_group *> &order) {
    std::vector<std::pair<size_t, size_t>> out;
    size_t b = 0;
    while (b < order.size()) {
        size_t e = b;
        std::vector<std::pair<const void *, int>> seen;
        while (e < order.size() && e - b < (size_t)kMaxGemmGroups) {
            const std::pair<const void *, int> key{order[e]->x, order[e]->n};
            if (std::find(seen.begin(), seen.end(), key) == seen.end()) {
                if (seen.size() == (size_t)kMaxInputs) break;
                seen.push_back(key);
            }
            ++e;
        }
        out.push_back({b, e});
        b = e;
    }
    return out;
}

}  // namespace
}  // namespace lamq

using namespace lamq;

static_assert(sizeof(lamq_gemm_group) == 104, "lamq_gemm_group is 104 bytes in the C ABI");

extern "C" size_t lamq_trellis_gemm_workspace_size(const lamq_gemm_group *groups, int ngroups, int64_t nvec) {
    if (groups == nullptr || ngroups <= 0 || nvec < kDecodeOnceVectors) return 0;
    size_t most = 0;
    std::vector<const lamq_gemm_group *> order;
    for (int i = 0; i < ngroups; ++i)
        if (groups[i].rows > 0 && groups[i].n > 0) order.push_back(&groups[i]);
    std::stable_sort(order.begin(), order.end(),
                     [](const lamq_gemm_group *a, const lamq_gemm_group *b) { return a->n > b->n; });
    for (const auto &be : batches(order)) {
        size_t bytes = 0;
        for (size_t i = be.first; i < be.second; ++i)
            bytes += (size_t)order[i]->rows * (size_t)decoded_ld(order[i]->n) * 2;
        most = std::max(most, bytes);
    }
    return most;
}

extern "C" int lamq_trellis_gemm(const lamq_gemm_group *groups, int ngroups, int64_t nvec, int y_bf16,
                                 void *workspace, size_t workspace_bytes, int *status, lamq_stream_t stream) {
    LAMQ_REQUIRE(ngroups >= 0 && nvec >= 0, "lamq_trellis_gemm: bad shape");
    if (ngroups == 0 || nvec == 0) return LAMQ_OK;
    LAMQ_REQUIRE(groups && status, "lamq_trellis_gemm: null pointer");
    std::vector<const lamq_gemm_group *> order;
    const int st0 = check_groups(groups, ngroups, nvec, order);
    if (st0) return st0;
    const size_t need = lamq_trellis_gemm_workspace_size(groups, ngroups, nvec);
    LAMQ_REQUIRE(workspace_bytes >= need && (need == 0 || (workspace && (uintptr_t)workspace % 16 == 0)),
                 "lamq_trellis_gemm: workspace of %zu bytes (16-byte aligned) needed, %zu given", need,
                 workspace_bytes);
    cudaStream_t s = (cudaStream_t)stream;
    for (const auto &be : batches(order)) {  // batches share the workspace: same stream, one after the other
        const int st = run_gemm(order.data() + be.first, (int)(be.second - be.first), nvec, y_bf16,
                                reinterpret_cast<uint16_t *>(workspace), status, s);
        if (st) return st;
    }
    return LAMQ_OK;
}
