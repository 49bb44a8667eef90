// Viterbi over the 12-bit bitshift trellis by a pair of warps (64 threads) per sequence, with packed fp32x2 arithmetic.
//
// The recursion is that of trellis_warp.cuh (opgraph/codes.py:151-181 restated over "best" arrays):
//   cost_t[s] = best_t[s >> k] + (x_t − C[s])²,   best_t[r] = min_{h < 2^k} cost_{t−1}[h·R + r]   (smallest h on ties)
// Thread p (0..63) of the pair owns RT = R/64 consecutive r and keeps the 64 table values C[h·R + r] of its
// predecessors in registers as fp32 pairs (half the registers of one warp per row, so twice the warps fit on an SM).
// (x − C) and its add to the best predecessor cost are computed two states at a time with sub/add.rn.f32x2 (states r
// and r + 1 share their predecessors), the square with two scalar mul.rn: every value is rounded exactly as the
// reference's scalar fp32 sub, mul and add (never fused). The minimum over the 2^k predecessors is a knock-out tournament (for
// k >= 3 two states at a time on packed differences) whose decisions are the sign bits of fp32 differences (the fp32
// pipe, not the half-rate compare/select pipe); the winner's k index bits are assembled from them by bit selects and
// appended to one back-pointer word per thread per step, so the traceback reads each step's choice with one shift. The pair exchanges the R best values through shared memory
// (double buffered, one named barrier per step), stored in 16-byte units swizzled by writer thread so that writes and
// reads are free of bank conflicts for every k.
#pragma once

#include "lamq_common.cuh"

namespace lamq {

template <int K>
struct PairTrellis {
    static constexpr int NB = 1 << K;
    static constexpr int R = 1 << (12 - K);
    static constexpr int RT = R / 64;                           // r values per thread
    static constexpr int DIST = (RT >> K) > 0 ? (RT >> K) : 1;  // distinct best values a thread reads per h
    static constexpr int UNITS = RT / 4;                        // 16-byte units a thread writes
    static constexpr int SH = (UNITS >= 8) ? 3 : (UNITS == 4) ? 2 : (UNITS == 2) ? 1 : 0;
    static constexpr int NBITS = RT * K;                        // back-pointer bits per thread per step (64K/NB <= 32)
    static constexpr int WORDS = 1;
    static_assert(NB * RT == 64, "each thread covers 64 predecessor states");
    static_assert(NBITS <= 32, "one back-pointer word per thread per step");
};

template <int K>
__device__ __forceinline__ int pslot(int r) {
    if constexpr (PairTrellis<K>::UNITS <= 1) {
        return r;
    } else {
        int u = r >> 2;
        u ^= (u >> PairTrellis<K>::SH) & 7;  // a bijection for SH >= 1
        return (u << 2) | (r & 3);
    }
}

typedef unsigned long long u64;

__device__ __forceinline__ u64 pk2(float lo, float hi) {
    u64 r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void upk2(u64 v, float &lo, float &hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ u64 sub2(u64 a, u64 b) {
    u64 r;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ u64 add2(u64 a, u64 b) {
    u64 r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}

// (d_lo², d_hi²), each square rounded by itself with the scalar multiply (mul.rn.f32, which is never contracted).
// A packed multiply — and a packed fma with a −0 addend — was fused with the add that follows into one rounding,
// which moved rare near-ties away from the reference's separately rounded fp32 cost (found by comparing a full table
// fit against the one-warp kernel, whose intrinsics the reference's paths match).
__device__ __forceinline__ u64 sq2(u64 d) {
    float lo, hi;
    upk2(d, lo, hi);
    return pk2(__fmul_rn(lo, lo), __fmul_rn(hi, hi));
}

__device__ __forceinline__ void pair_sync(int bar) { asm volatile("bar.sync %0, 64;" ::"r"(bar) : "memory"); }

// cv[h][j] = (C[h·R + p·RT + 2j], C[h·R + p·RT + 2j + 1]) as fp32 (from an fp32 table, or rounded from the fp64 one
// like values.float()).
template <int K, typename TT>
__device__ __forceinline__ void load_pair_values(const TT *__restrict__ table, int p,
                                                 u64 (&cv)[PairTrellis<K>::NB][PairTrellis<K>::RT / 2]) {
    using T = PairTrellis<K>;
#pragma unroll
    for (int h = 0; h < T::NB; ++h)
#pragma unroll
        for (int j = 0; j < T::RT / 2; ++j) {
            const int s = h * T::R + p * T::RT + 2 * j;
            cv[h][j] = pk2((float)__ldg(table + s), (float)__ldg(table + s + 1));
        }
}

template <int K>
__device__ __forceinline__ void init_best_pair(float *best, int p, bool has_start, int start) {
    using T = PairTrellis<K>;
    const int r0 = start & (T::R - 1);
    const float inf = __int_as_float(0x7f800000);
#pragma unroll
    for (int i = 0; i < T::RT; i += 4) {
        const int r = p * T::RT + i;
        float4 v;
        v.x = (!has_start || r + 0 == r0) ? 0.f : inf;
        v.y = (!has_start || r + 1 == r0) ? 0.f : inf;
        v.z = (!has_start || r + 2 == r0) ? 0.f : inf;
        v.w = (!has_start || r + 3 == r0) ? 0.f : inf;
        *reinterpret_cast<float4 *>(best + pslot<K>(r)) = v;
    }
}

// Decision words: the sign bit of c_b − c_a is set exactly when c_b < c_a (for these non-negative costs the rounded
// difference has the sign of the exact one; ties and inf − inf give 0, keeping a). The tournament carries, for each
// surviving slot, the sign-bit words of its winner's index bits: a later level's decision selects between the two
// halves' words bit by bit (one LOP3 each), so at the end the K bits of the winning predecessor h are known and are
// appended (most significant first) to the thread's back-pointer word by funnel shifts — K bits per r, one word per
// step, decoded on the traceback with a single shift.
__device__ __forceinline__ uint32_t sel_bits(uint32_t e, uint32_t right, uint32_t left) {
    return (e & right) | (~e & left);  // bit 31: right's when the right side won
}

// Knock-out minimum of NB costs (pairs, then pairs of winners, …), the left (smaller h) winning ties: the first
// minimum, as torch.min picks it. Appends the winner's K index bits to `word`.
template <int K>
__device__ __forceinline__ float tournament(float (&m)[PairTrellis<K>::NB], uint32_t &word) {
    constexpr int NB = PairTrellis<K>::NB;
    uint32_t idx[NB / 2][K];
    int lvl = 0;
#pragma unroll
    for (int n = NB; n > 1; n >>= 1, ++lvl) {
#pragma unroll
        for (int g = 0; g < n / 2; ++g) {
            const uint32_t e = __float_as_uint(__fsub_rn(m[2 * g + 1], m[2 * g]));
#pragma unroll
            for (int b = 0; b < lvl; ++b) idx[g][b] = sel_bits(e, idx[2 * g + 1][b], idx[2 * g][b]);
            idx[g][lvl] = e;
            m[g] = fminf(m[2 * g], m[2 * g + 1]);
        }
    }
#pragma unroll
    for (int b = K - 1; b >= 0; --b) word = __funnelshift_l(idx[0][b], word, 1);
    return m[0];
}

// Whether the two states r, r + 1 of a pair run their tournaments together (tournament2): faster for 8 and 16
// predecessors, slower for 2 and 4 (measured on B200).
template <int K>
constexpr bool kPairedTournament = K >= 3;

// The tournament for the two states r and r + 1 at once (m[h] holds their costs as an fp32 pair): one packed
// subtraction gives both states' differences (each rounded as the scalar fp32 subtraction). Appends r's K index bits,
// then r + 1's.
template <int K>
__device__ __forceinline__ u64 tournament2(u64 (&m)[PairTrellis<K>::NB], uint32_t &word) {
    constexpr int NB = PairTrellis<K>::NB;
    uint32_t ilo[NB / 2][K], ihi[NB / 2][K];
    int lvl = 0;
#pragma unroll
    for (int n = NB; n > 1; n >>= 1, ++lvl) {
#pragma unroll
        for (int g = 0; g < n / 2; ++g) {
            float dlo, dhi, alo, ahi, blo, bhi;
            upk2(sub2(m[2 * g + 1], m[2 * g]), dlo, dhi);
            const uint32_t elo = __float_as_uint(dlo), ehi = __float_as_uint(dhi);
#pragma unroll
            for (int b = 0; b < lvl; ++b) {
                ilo[g][b] = sel_bits(elo, ilo[2 * g + 1][b], ilo[2 * g][b]);
                ihi[g][b] = sel_bits(ehi, ihi[2 * g + 1][b], ihi[2 * g][b]);
            }
            ilo[g][lvl] = elo;
            ihi[g][lvl] = ehi;
            upk2(m[2 * g], alo, ahi);
            upk2(m[2 * g + 1], blo, bhi);
            m[g] = pk2(fminf(alo, blo), fminf(ahi, bhi));
        }
    }
#pragma unroll
    for (int b = K - 1; b >= 0; --b) word = __funnelshift_l(ilo[0][b], word, 1);
#pragma unroll
    for (int b = K - 1; b >= 0; --b) word = __funnelshift_l(ihi[0][b], word, 1);
    return m[0];
}

// One add-compare-select step for the thread's RT values of r: best_t into bout, the decision bits into words.
template <int K>
__device__ __forceinline__ void acs_pair(const float *__restrict__ bin, float *__restrict__ bout, float xp, int p,
                                         const u64 (&cv)[PairTrellis<K>::NB][PairTrellis<K>::RT / 2],
                                         uint32_t (&words)[PairTrellis<K>::WORDS]) {
    using T = PairTrellis<K>;
    constexpr int CH = (T::DIST >= 4) ? 4 : 1;                // best values loaded per chunk per h
    constexpr int CI = (T::DIST >= 4) ? (4 << K) : T::RT;     // r values per chunk
    const u64 xx = pk2(xp, xp);
#pragma unroll
    for (int w = 0; w < T::WORDS; ++w) words[w] = 0u;
#pragma unroll
    for (int c0 = 0; c0 < T::RT; c0 += CI) {
        float bv[T::NB][CH];
#pragma unroll
        for (int h = 0; h < T::NB; ++h) {
            const int base = h * (T::R >> K) + ((p * T::RT + c0) >> K);
            if constexpr (CH == 4) {
                const float4 v = *reinterpret_cast<const float4 *>(bin + pslot<K>(base));
                bv[h][0] = v.x; bv[h][1] = v.y; bv[h][2] = v.z; bv[h][3] = v.w;
            } else {
                bv[h][0] = bin[pslot<K>(base)];
            }
        }
        // r = ii and ii + 1 share their predecessors' best values (ii >> K), so the add is paired too
        u64 bb[T::NB][CH];
#pragma unroll
        for (int h = 0; h < T::NB; ++h)
#pragma unroll
            for (int j = 0; j < CH; ++j) bb[h][j] = pk2(bv[h][j], bv[h][j]);
        float nb4[4];
#pragma unroll
        for (int i = 0; i < CI; i += 2) {
            const int ii = c0 + i;
            u64 c2[T::NB];
#pragma unroll
            for (int h = 0; h < T::NB; ++h) {
                const u64 d = sub2(xx, cv[h][ii >> 1]);  // (x − C) for r = ii and ii + 1
                c2[h] = add2(bb[h][(CH == 4) ? (i >> K) : 0], sq2(d));  // best + (x − C)²
            }
            if constexpr (kPairedTournament<K>) {
                upk2(tournament2<K>(c2, words[0]), nb4[i & 3], nb4[(i & 3) + 1]);
            } else {
                float clo[T::NB], chi[T::NB];
#pragma unroll
                for (int h = 0; h < T::NB; ++h) upk2(c2[h], clo[h], chi[h]);
                nb4[i & 3] = tournament<K>(clo, words[0]);
                nb4[(i & 3) + 1] = tournament<K>(chi, words[0]);
            }
            if ((i & 3) == 2)
                *reinterpret_cast<float4 *>(bout + pslot<K>(p * T::RT + ii - 2)) =
                    make_float4(nb4[0], nb4[1], nb4[2], nb4[3]);
        }
    }
}

// The chosen predecessor h of r at a step: the owner thread's K bits for its i-th r (args: 64 words, one per thread).
template <int K>
__device__ __forceinline__ int decode_choice(const uint32_t *__restrict__ args, int r) {
    using T = PairTrellis<K>;
    const int owner = r / T::RT, i = r % T::RT;
    return (int)((args[owner] >> (T::NBITS - K - i * K)) & (uint32_t)(T::NB - 1));
}

// First state of minimum final cost over the pair (smallest state on ties); red holds 4 words of pair scratch.
template <int K>
__device__ __forceinline__ int final_argmin_pair(const float *__restrict__ best, float xl, int p, int bar,
                                                 const u64 (&cv)[PairTrellis<K>::NB][PairTrellis<K>::RT / 2],
                                                 float *red) {
    using T = PairTrellis<K>;
    const u64 xx = pk2(xl, xl);
    float m = __int_as_float(0x7f800000);
    int ms = 0x7fffffff;
#pragma unroll
    for (int h = 0; h < T::NB; ++h) {
#pragma unroll
        for (int i = 0; i < T::RT; i += 2) {
            const float b = best[pslot<K>(h * (T::R >> K) + ((p * T::RT + i) >> K))];
            const u64 d = sub2(xx, cv[h][i >> 1]);
            const u64 c = add2(pk2(b, b), sq2(d));
            float lo, hi;
            upk2(c, lo, hi);
            const int s = h * T::R + p * T::RT + i;  // states visited in increasing order
            if (lo < m || ms == 0x7fffffff) { m = lo; ms = s; }
            if (hi < m) { m = hi; ms = s + 1; }
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float om = __shfl_xor_sync(0xffffffffu, m, off);
        const int os = __shfl_xor_sync(0xffffffffu, ms, off);
        if (om < m || (om == m && os < ms)) { m = om; ms = os; }
    }
    const int w = p >> 5;
    if ((p & 31) == 0) {
        red[2 * w] = m;
        reinterpret_cast<int *>(red)[2 * w + 1] = ms;
    }
    pair_sync(bar);
    const float m0 = red[0], m1 = red[2];
    const int s0 = reinterpret_cast<int *>(red)[1], s1 = reinterpret_cast<int *>(red)[3];
    const int fs = (m1 < m0 || (m1 == m0 && s1 < s0)) ? s1 : s0;
    pair_sync(bar);  // red is reused by the next window
    return fs;
}

// Decodes one window x_0..x_{T−1} (lane t of each warp holds x_t, T <= 32) with the pair; lane t of the pair's first
// warp returns the state at position t. best0/best1: two R-float buffers; args: T x WORDS x 64 words; red: 4 words.
template <int K>
__device__ __forceinline__ int viterbi_window_pair(float xv, int T, int start, int p, int bar,
                                                   const u64 (&cv)[PairTrellis<K>::NB][PairTrellis<K>::RT / 2],
                                                   float *best0, float *best1, uint32_t *args, float *red) {
    using Tr = PairTrellis<K>;
    init_best_pair<K>(best0, p, true, start);
    pair_sync(bar);
    float *bin = best0, *bout = best1;
    for (int t = 1; t < T; ++t) {
        const float xp = __shfl_sync(0xffffffffu, xv, t - 1);
        uint32_t words[Tr::WORDS];
        acs_pair<K>(bin, bout, xp, p, cv, words);
#pragma unroll
        for (int w = 0; w < Tr::WORDS; ++w) args[(t * Tr::WORDS + w) * 64 + p] = words[w];
        pair_sync(bar);
        float *tmp = bin;
        bin = bout;
        bout = tmp;
    }
    const float xl = __shfl_sync(0xffffffffu, xv, T - 1);
    const int fs = final_argmin_pair<K>(bin, xl, p, bar, cv, red);
    if (p >= 32) return 0;  // only the first warp needs the path
    // traceback: every lane walks the path (broadcast reads); lane t keeps position t
    const int lane = p & 31;
    int s = fs;
    int mine = (lane == T - 1) ? s : 0;
    for (int t = T - 1; t > 0; --t) {
        const int r = s >> K;
        s = decode_choice<K>(args + t * Tr::WORDS * 64, r) * Tr::R + r;
        if (lane == t - 1) mine = s;
    }
    return mine;
}

}  // namespace lamq
