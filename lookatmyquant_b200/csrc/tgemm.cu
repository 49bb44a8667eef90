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
// Tiles: 128 weight rows (the MMA's M, TMEM lanes) × 256 input vectors (N, one accumulator of 256 TMEM columns),
// K in slices of 64. A work unit is (row tile, block of NACC·256 vectors); with NACC = 2 both accumulators share each
// decoded slice (the decode is amortised over 512 vectors), with NACC = 1 they alternate between units so the
// epilogue of one unit overlaps the next unit's MMAs.
//
// Warp roles (320 threads): warp 0 issues the TMA loads of X (K-major, 128-byte swizzle), warp 1 allocates TMEM and
// issues the MMAs (one thread), warps 2-5 decode (thread d owns row d of the tile: it reads the row's stream words
// for the slice — prefetched one slice ahead — cuts the 64 states out with funnel shifts, looks them up in its warp's
// bf16 copy of the table and stores the 64 bf16 values as eight 16-byte chunks in the 128-byte-swizzled K-major
// layout the MMA descriptor reads), warps 6-9 drain the accumulators (row scale, optional map, fp32 or bf16 out).
// Every wait is bounded (2 s): a timeout sets the status word and the CTA winds down.
#include <algorithm>

#include <cuda.h>
#include <cuda_bf16.h>

#include "lamq_common.cuh"
#include "sm100.cuh"

namespace lamq {
namespace {

using namespace sm100;

constexpr int TM = 128, TN = 256, TK = 64;
constexpr int A_BYTES = TM * TK * 2, B_BYTES = TN * TK * 2;
constexpr int kDecWarps = 4, kEpiWarps = 4;
constexpr int kThreads = (2 + kDecWarps + kEpiWarps) * 32;
constexpr uint32_t kTmemCols = 512;
constexpr int kTableEntries = 4096;
constexpr int kMaxGemmGroups = 16;

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
    int64_t first;           // first row tile of the group in the launch's numbering
};

struct GemmParams {
    GemmGroup g[kMaxGemmGroups];
    int ng;
    int n, kslices, bn;      // bn: vectors per accumulator (<= 256, a multiple of 16)
    int64_t nvec;
    int64_t tiles, units;    // row tiles of all groups; units = tiles x vector blocks
    int y_bf16;
    int *status;
};

template <int NACC>
struct Layout {
    static constexpr int STAGES = NACC == 2 ? 2 : 4;
    static constexpr int STAGE_BYTES = A_BYTES + NACC * B_BYTES;
    static constexpr int TABLE_OFF = STAGES * STAGE_BYTES;
    static constexpr int BAR_OFF = TABLE_OFF + kDecWarps * kTableEntries * 2;
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

// Unit u: vector block u / tiles, row tile u % tiles (consecutive units share the vector block, which stays in L2).
__device__ __forceinline__ void unit_of(const GemmParams &p, int64_t u, int &vb, int &g, int64_t &rt) {
    vb = (int)(u / p.tiles);
    const int64_t t = u % p.tiles;
    g = 0;
    while (g + 1 < p.ng && p.g[g + 1].first <= t) ++g;
    rt = t - p.g[g].first;
}

// Stream words of one row for the slice starting at column c0: bits [(N − c0 − 64)·K, +64K+12) (word-aligned).
template <int K>
struct Slice {
    static constexpr int NW = (63 * K + 12 + 31) / 32;
    uint32_t w[NW];
};

template <int K>
__device__ __forceinline__ void load_slice(Slice<K> &s, const uint32_t *row, int wpr, int N, int c0, bool live) {
    const int wb = ((N - c0 - 64) * K) >> 5;  // may be negative for a last slice of 32 columns
#pragma unroll
    for (int q = 0; q < Slice<K>::NW; ++q) {
        const int w = wb + q;
        s.w[q] = (live && w >= 0 && w < wpr) ? __ldg(row + w) : 0u;
    }
}

__device__ __forceinline__ uint32_t bf16_pair(const uint16_t *tab, uint32_t s0, uint32_t s1) {
    return (uint32_t)tab[s0] | ((uint32_t)tab[s1] << 16);
}

// Decodes the 64 states of a slice (column c0 + i at stream offset (63 − i)·K) and stores the bf16 row.
template <int K>
__device__ __forceinline__ void store_slice_packed(const Slice<K> &s, const uint16_t *tab, uint32_t lmask,
                                                   uint32_t arow, int swz, int valid) {
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        uint32_t pk[4];
#pragma unroll
        for (int h = 0; h < 4; ++h) {
            uint32_t st[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int i = 8 * c + 2 * h + e;
                const int o = (63 - i) * K;
                st[e] = __funnelshift_r(s.w[o >> 5], s.w[(o >> 5) + 1], o & 31) & lmask;
            }
            pk[h] = bf16_pair(tab, st[0], st[1]);
            if (8 * c + 2 * h >= valid) pk[h] = 0u;
            else if (8 * c + 2 * h + 1 >= valid) pk[h] &= 0xFFFFu;
        }
        sts128(arow + ((uint32_t)(c ^ swz) << 4), pk[0], pk[1], pk[2], pk[3]);
    }
}

__device__ __forceinline__ void store_slice_states(const uint4 (&v)[8], const uint16_t *tab, uint32_t lmask,
                                                   uint32_t arow, int swz, int valid) {
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        const uint32_t raw[4] = {v[c].x, v[c].y, v[c].z, v[c].w};
        uint32_t pk[4];
#pragma unroll
        for (int h = 0; h < 4; ++h) {
            pk[h] = bf16_pair(tab, raw[h] & lmask, (raw[h] >> 16) & lmask);
            if (8 * c + 2 * h >= valid) pk[h] = 0u;
            else if (8 * c + 2 * h + 1 >= valid) pk[h] &= 0xFFFFu;
        }
        sts128(arow + ((uint32_t)(c ^ swz) << 4), pk[0], pk[1], pk[2], pk[3]);
    }
}

__device__ __forceinline__ void load_states(uint4 (&v)[8], const int16_t *row, int c0, int n, bool live) {
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        const int j = c0 + 8 * c;
        v[c] = (live && j < n) ? __ldg(reinterpret_cast<const uint4 *>(row + j)) : make_uint4(0, 0, 0, 0);
    }
}

// The decode of one unit's slices by decoder thread d (row d of the tile). Returns false on a timeout.
template <int K, int NACC>
__device__ bool decode_unit(const GemmParams &p, const GemmGroup &g, int64_t rt, int d, const uint16_t *tab,
                            uint32_t smem_base, uint32_t full0, uint32_t empty0, int &stage, uint32_t &phase) {
    using LY = Layout<NACC>;
    const int64_t row = rt * TM + d;
    const bool live = row < g.rows;
    const uint32_t lmask = (1u << g.L) - 1u;
    const int swz = d & 7;
    const int lane = threadIdx.x & 31;
    const int n = p.n;
    if constexpr (K == 0) {
        const int16_t *srow = g.states + (live ? row : 0) * g.lds;
        uint4 cur[8], nxt[8];
        load_states(cur, srow, 0, n, live);
        for (int kb = 0; kb < p.kslices; ++kb) {
            if (kb + 1 < p.kslices) load_states(nxt, srow, (kb + 1) * TK, n, live);
            if (!mbar_wait(empty0 + 8 * stage, phase ^ 1, p.status)) return false;
            const uint32_t arow = smem_base + stage * LY::STAGE_BYTES + d * 128;
            store_slice_states(cur, tab, lmask, arow, swz, live ? n - kb * TK : 0);
            fence_async_shared();
            __syncwarp();
            if (lane == 0) mbar_arrive(full0 + 8 * stage);
            if (++stage == LY::STAGES) {
                stage = 0;
                phase ^= 1;
            }
#pragma unroll
            for (int c = 0; c < 8; ++c) cur[c] = nxt[c];
        }
    } else {
        const int N = (n + 31) / 32 * 32;
        const int wpr = N / 32 * K;
        const uint32_t *crow = g.codes + (live ? row : 0) * (int64_t)wpr;
        Slice<K> cur, nxt;
        load_slice<K>(cur, crow, wpr, N, 0, live);
        for (int kb = 0; kb < p.kslices; ++kb) {
            if (kb + 1 < p.kslices) load_slice<K>(nxt, crow, wpr, N, (kb + 1) * TK, live);
            if (!mbar_wait(empty0 + 8 * stage, phase ^ 1, p.status)) return false;
            const uint32_t arow = smem_base + stage * LY::STAGE_BYTES + d * 128;
            store_slice_packed<K>(cur, tab, lmask, arow, swz, live ? n - kb * TK : 0);
            fence_async_shared();
            __syncwarp();
            if (lane == 0) mbar_arrive(full0 + 8 * stage);
            if (++stage == LY::STAGES) {
                stage = 0;
                phase ^= 1;
            }
            cur = nxt;
        }
    }
    return true;
}

template <int NACC>
__global__ void __launch_bounds__(kThreads, 1)
    trellis_gemm_kernel(const __grid_constant__ CUtensorMap mapX, const __grid_constant__ GemmParams p) {
    using LY = Layout<NACC>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + LY::BAR_OFF);
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 2 * LY::STAGES + 5);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t smem_base = smem_u32(smem);
    const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + LY::STAGES);
    const uint32_t tfull0 = smem_u32(bars + 2 * LY::STAGES), tempty0 = smem_u32(bars + 2 * LY::STAGES + 2);
    const uint32_t drain = smem_u32(bars + 2 * LY::STAGES + 4);
    if (threadIdx.x == 0) {
        for (int s = 0; s < LY::STAGES; ++s) {
            mbar_init(full0 + 8 * s, 1 + kDecWarps);  // the TMA's expect_tx arrival + one per decoder warp
            mbar_init(empty0 + 8 * s, 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(tfull0 + 8 * a, 1);
            mbar_init(tempty0 + 8 * a, kEpiWarps * 32);
        }
        mbar_init(drain, 1);
        fence_mbar_init();
        prefetch_tmap(&mapX);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_holder), kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;
    const int bn = p.bn;
    const uint32_t b_tx = (uint32_t)bn * TK * 2;

    if (warp == 0) {
        if (lane == 0) {  // ---- TMA producer: X slices of NACC blocks of bn vectors
            int stage = 0;
            uint32_t phase = 0;
            int64_t issued = 0;
            bool ok = true;
            for (int64_t u = blockIdx.x; ok && u < p.units; u += gridDim.x) {
                int vb, g;
                int64_t rt;
                unit_of(p, u, vb, g, rt);
                for (int kb = 0; kb < p.kslices; ++kb) {
                    if (!mbar_wait(empty0 + 8 * stage, phase ^ 1, p.status)) {
                        ok = false;
                        break;
                    }
                    const uint32_t fb = full0 + 8 * stage;
                    mbar_expect_tx(fb, NACC * b_tx);
                    const uint32_t sb = smem_base + stage * LY::STAGE_BYTES + A_BYTES;
#pragma unroll
                    for (int j = 0; j < NACC; ++j)
                        tma_load_2d(sb + j * B_BYTES, &mapX, kb * TK, (vb * NACC + j) * bn, fb);
                    ++issued;
                    if (++stage == LY::STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            if (!ok) {  // let the copies in flight land before the CTA exits
                const int64_t outstanding = issued < LY::STAGES ? issued : LY::STAGES;
                for (int64_t i = issued - outstanding; i < issued; ++i) {
                    const int s = (int)(i % LY::STAGES);
                    const uint32_t ph = (uint32_t)((i / LY::STAGES) & 1);
                    const unsigned long long t0 = globaltimer();
                    while (!mbar_try_wait(full0 + 8 * s, ph) && globaltimer() - t0 < kWaitTimeoutNs) {
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {  // ---- MMA issuer
            const uint32_t idesc = idesc_bf16_f32(TM, bn, false, false);
            int stage = 0;
            uint32_t phase = 0;
            uint32_t uses[2] = {0, 0};
            int64_t it = 0;
            bool ok = true;
            for (int64_t u = blockIdx.x; ok && u < p.units; u += gridDim.x, ++it) {
                int slot[NACC];
#pragma unroll
                for (int j = 0; j < NACC; ++j) {
                    slot[j] = NACC == 2 ? j : (int)(it & 1);
                    if (!mbar_wait(tempty0 + 8 * slot[j], (uses[slot[j]] & 1) ^ 1, p.status)) ok = false;
                    ++uses[slot[j]];
                }
                if (!ok) break;
                tc_fence_after();
                for (int kb = 0; kb < p.kslices; ++kb) {
                    if (!mbar_wait(full0 + 8 * stage, phase, p.status)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = smem_base + stage * LY::STAGE_BYTES, sb = sa + A_BYTES;
#pragma unroll
                    for (int j = 0; j < NACC; ++j) {
#pragma unroll
                        for (int kk = 0; kk < TK / 16; ++kk) {
                            const uint64_t ad = smem_desc_sw128(sa + kk * 32, 16, 1024);
                            const uint64_t bd = smem_desc_sw128(sb + j * B_BYTES + kk * 32, 16, 1024);
                            mma_f16_ss(tmem + slot[j] * TN, ad, bd, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
                        }
                    }
                    mma_commit(empty0 + 8 * stage);
                    if (++stage == LY::STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (!ok) break;
#pragma unroll
                for (int j = 0; j < NACC; ++j) mma_commit(tfull0 + 8 * slot[j]);
            }
            mma_commit(drain);
            const unsigned long long t0 = globaltimer();
            while (!mbar_try_wait(drain, 0) && globaltimer() - t0 < kWaitTimeoutNs) {
            }
        }
    } else if (warp < 2 + kDecWarps) {  // ---- decoders: thread d owns row d of the tile
        const int dw = warp - 2, d = threadIdx.x - 64;
        uint16_t *tab = reinterpret_cast<uint16_t *>(smem + LY::TABLE_OFF) + dw * kTableEntries;
        int stage = 0;
        uint32_t phase = 0;
        int cur_group = -1;
        for (int64_t u = blockIdx.x; u < p.units; u += gridDim.x) {
            int vb, gi;
            int64_t rt;
            unit_of(p, u, vb, gi, rt);
            const GemmGroup &g = p.g[gi];
            if (gi != cur_group) {  // this warp's copy of the group's table, as bf16
                __syncwarp();
                const int nt = 1 << g.L;
                for (int i = lane; i < kTableEntries; i += 32) {
                    const float v = i < nt ? __ldg(g.table + i) : 0.f;
                    tab[i] = __bfloat16_as_ushort(__float2bfloat16_rn(v));
                }
                __syncwarp();
                cur_group = gi;
            }
            bool ok;
            switch (g.states ? 0 : g.k) {
                case 0: ok = decode_unit<0, NACC>(p, g, rt, d, tab, smem_base, full0, empty0, stage, phase); break;
                case 1: ok = decode_unit<1, NACC>(p, g, rt, d, tab, smem_base, full0, empty0, stage, phase); break;
                case 2: ok = decode_unit<2, NACC>(p, g, rt, d, tab, smem_base, full0, empty0, stage, phase); break;
                case 3: ok = decode_unit<3, NACC>(p, g, rt, d, tab, smem_base, full0, empty0, stage, phase); break;
                default: ok = decode_unit<4, NACC>(p, g, rt, d, tab, smem_base, full0, empty0, stage, phase); break;
            }
            if (!ok) break;
        }
    } else {  // ---- epilogue: warp w reads TMEM lanes 32·(w % 4).. (rows of the tile)
        const int q = warp & 3;
        uint32_t uses[2] = {0, 0};
        int64_t it = 0;
        bool ok = true;
        for (int64_t u = blockIdx.x; ok && u < p.units; u += gridDim.x, ++it) {
            int vb, gi;
            int64_t rt;
            unit_of(p, u, vb, gi, rt);
            const GemmGroup &g = p.g[gi];
            const int64_t row = rt * TM + 32 * q + lane;
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
                mbar_arrive(tempty0 + 8 * slot);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, kTmemCols);
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

template <int NACC>
int launch_gemm(const CUtensorMap &map, const GemmParams &p, cudaStream_t s) {
    const cudaError_t e = smem_limit_once((const void *)trellis_gemm_kernel<NACC>, (int)Layout<NACC>::SMEM);
    if (e != cudaSuccess) {
        set_error("lamq_trellis_gemm: %s", cudaGetErrorString(e));
        return LAMQ_ERR_CUDA;
    }
    const int64_t grid = std::min<int64_t>(p.units, num_sms());
    trellis_gemm_kernel<NACC><<<(unsigned)grid, kThreads, Layout<NACC>::SMEM, s>>>(map, p);
    LAMQ_CHECK_LAUNCH("lamq_trellis_gemm");
    return LAMQ_OK;
}

// One launch over up to kMaxGemmGroups groups that read the same X.
int run_gemm(const lamq_gemm_group *groups, int ngroups, int n, const uint16_t *x, int64_t ldx, int64_t nvec,
             int y_bf16, int *status, cudaStream_t s) {
    EncodeTiled enc = encode_fn();
    if (enc == nullptr) {
        set_error("lamq_trellis_gemm: cuTensorMapEncodeTiled is unavailable");
        return LAMQ_ERR_CUDA;
    }
    const int nacc = nvec > TN ? 2 : 1;
    const int bn = nvec >= TN ? TN : (int)((nvec + 15) / 16 * 16);
    CUtensorMap map;
    cuuint64_t dims[2] = {(cuuint64_t)n, (cuuint64_t)nvec};
    cuuint64_t strides[1] = {(cuuint64_t)ldx * 2};
    cuuint32_t box[2] = {(cuuint32_t)TK, (cuuint32_t)bn};
    cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t *>(x), dims, strides, box,
                           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("lamq_trellis_gemm: cuTensorMapEncodeTiled failed (%d)", (int)r);
        return LAMQ_ERR_INVALID;
    }
    GemmParams p{};
    p.n = n;
    p.kslices = (n + TK - 1) / TK;
    p.bn = bn;
    p.nvec = nvec;
    p.y_bf16 = y_bf16;
    p.status = status;
    int64_t tiles = 0;
    int ng = 0;
    for (int i = 0; i < ngroups; ++i) {
        const lamq_gemm_group &g = groups[i];
        if (g.rows == 0) continue;
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
        d.first = tiles;
        tiles += (g.rows + TM - 1) / TM;
    }
    if (ng == 0) return LAMQ_OK;
    p.ng = ng;
    p.tiles = tiles;
    const int64_t vblocks = (nvec + (int64_t)nacc * bn - 1) / ((int64_t)nacc * bn);
    p.units = tiles * vblocks;
    return nacc == 2 ? launch_gemm<2>(map, p, s) : launch_gemm<1>(map, p, s);
}

}  // namespace
}  // namespace lamq

using namespace lamq;

static_assert(sizeof(lamq_gemm_group) == 80, "lamq_gemm_group is 80 bytes in the C ABI");

extern "C" int lamq_trellis_gemm(const lamq_gemm_group *groups, int ngroups, int n, const uint16_t *x, int64_t ldx,
                                 int64_t nvec, int y_bf16, int *status, lamq_stream_t stream) {
    LAMQ_REQUIRE(ngroups >= 0 && n > 0 && nvec >= 0 && ldx >= n, "lamq_trellis_gemm: bad shape");
    if (ngroups == 0 || nvec == 0) return LAMQ_OK;
    LAMQ_REQUIRE(groups && x && status, "lamq_trellis_gemm: null pointer");
    LAMQ_REQUIRE(ldx % 8 == 0 && ((uintptr_t)x % 16) == 0,
                 "lamq_trellis_gemm: x must be 16-byte aligned with a leading dimension that is a multiple of 8");
    for (int i = 0; i < ngroups; ++i) {
        const lamq_gemm_group &g = groups[i];
        LAMQ_REQUIRE(g.rows >= 0, "lamq_trellis_gemm: group %d has %lld rows", i, (long long)g.rows);
        if (g.rows == 0) continue;
        LAMQ_REQUIRE(g.scales && g.table && g.y, "lamq_trellis_gemm: group %d: null pointer", i);
        LAMQ_REQUIRE((g.codes != nullptr) != (g.states != nullptr),
                     "lamq_trellis_gemm: group %d: give packed codes or int16 states, not both", i);
        LAMQ_REQUIRE(g.L >= 1 && g.L <= 12, "lamq_trellis_gemm: group %d: L in 1..12 (got %d)", i, g.L);
        if (g.codes) {
            LAMQ_REQUIRE(g.k >= 1 && g.k <= 4 && g.L > g.k,
                         "lamq_trellis_gemm: group %d: packed widths k in 1..4 and L in k+1..12 (k %d, L %d)", i, g.k,
                         g.L);
        } else {
            LAMQ_REQUIRE(n % 8 == 0 && g.lds >= n && g.lds % 8 == 0 && ((uintptr_t)g.states % 16) == 0,
                         "lamq_trellis_gemm: group %d: int16 states need n and lds multiples of 8 and 16-byte rows", i);
        }
        LAMQ_REQUIRE(nvec <= 1 || g.ldy >= g.rows, "lamq_trellis_gemm: group %d: ldy %lld below its %lld rows", i,
                     (long long)g.ldy, (long long)g.rows);
    }
    cudaStream_t s = (cudaStream_t)stream;
    for (int b = 0; b < ngroups; b += kMaxGemmGroups) {
        const int st = run_gemm(groups + b, std::min(kMaxGemmGroups, ngroups - b), n, x, ldx, nvec, y_bf16, status, s);
        if (st) return st;
    }
    return LAMQ_OK;
}
