// Warp-level Viterbi over the 12-bit bitshift trellis: one warp decodes one sequence (a row's window).
//
// The recursion (opgraph/codes.py:151-181) is restated in terms of "best" arrays: with R = 2^(L-k) and nb = 2^k,
//   cost_t[s] = best_t[s >> k] + (x_t - C[s])^2           (codes.py:164,172: one fp32 sub, one mul, one add)
//   best_t[r] = min_{h < nb} cost_{t-1}[h·R + r]           (codes.py:170: the smallest h on ties)
// with best_0 = 0 everywhere (free start; 0 + d == d exactly) or 0 at the start state's successors' shared index
// start & (R-1) and +inf elsewhere (codes.py:165-167). The final state is the first minimum of cost_{T-1}
// (codes.py:173) and the back-pointers are followed to t = 0 (codes.py:174-179).
//
// Layout: lane l owns RL = R/32 consecutive r = l·RL + i. It keeps in registers the table values of its predecessor
// states C[h·R + r] (nb·RL = 128 values for every k: the warp covers all 4096 states), so a step touches shared memory
// only for the R best values (read as the predecessors' best_{t-1}[s >> k], written for the lane's own r) and one
// 64-bit word of packed back-pointers per lane. The best array lives in shared memory in 16-byte units swizzled by the
// writer lane (unit ^= (unit >> log2(units per lane)) & 7) so both the writes and the reads are free of bank conflicts
// (except a 2-way read conflict at k = 1).
#pragma once

#include "lamq_common.cuh"

namespace lamq {

constexpr int kL = 12;
constexpr int kStates = 1 << kL;

template <int K>
struct Trellis {
    static constexpr int NB = 1 << K;            // predecessors per state, successors per state
    static constexpr int R = 1 << (kL - K);      // distinct "r = s >> k" values
    static constexpr int RL = R / 32;            // r values per lane
    static constexpr int DIST = (RL >> K) > 0 ? (RL >> K) : 1;  // distinct best values a lane reads per h
    static constexpr int UNITS = RL / 4;         // 16-byte units a lane writes
    static constexpr int SH = (UNITS == 16) ? 4 : (UNITS == 8) ? 3 : (UNITS == 4) ? 2 : 1;
    static_assert(NB * RL == 128, "each lane covers 128 predecessor states");
};

// Swizzled float index of best[r].
template <int K>
__device__ __forceinline__ int best_slot(int r) {
    int u = r >> 2;
    u ^= (u >> Trellis<K>::SH) & 7;
    return (u << 2) | (r & 3);
}

// Loads the lane's predecessor table values: cv[h][i] = C[h·R + lane·RL + i] (fp32, rounded from the fp64 table as
// the reference's values.to(float32) does).
template <int K>
__device__ __forceinline__ void load_pred_values(const double *__restrict__ table, int lane,
                                                 float (&cv)[Trellis<K>::NB][Trellis<K>::RL]) {
    using Tr = Trellis<K>;
#pragma unroll
    for (int h = 0; h < Tr::NB; ++h)
#pragma unroll
        for (int i = 0; i < Tr::RL; ++i) cv[h][i] = (float)__ldg(table + h * Tr::R + lane * Tr::RL + i);
}

template <int K>
__device__ __forceinline__ void load_pred_values_f32(const float *__restrict__ table, int lane,
                                                     float (&cv)[Trellis<K>::NB][Trellis<K>::RL]) {
    using Tr = Trellis<K>;
#pragma unroll
    for (int h = 0; h < Tr::NB; ++h)
#pragma unroll
        for (int i = 0; i < Tr::RL; ++i) cv[h][i] = __ldg(table + h * Tr::R + lane * Tr::RL + i);
}

// Reads best_{t-1} values needed by lane `lane` for predecessor block h: DIST floats starting at r-index
// h·(R >> k) + (lane·RL) >> k.
template <int K>
__device__ __forceinline__ void read_best(const float *__restrict__ best, int lane, int h, float *out) {
    using Tr = Trellis<K>;
    const int base = h * (Tr::R >> K) + ((lane * Tr::RL) >> K);
    if constexpr (Tr::DIST >= 4) {
#pragma unroll
        for (int c = 0; c < Tr::DIST; c += 4) {
            float4 v = *reinterpret_cast<const float4 *>(best + best_slot<K>(base + c));
            out[c] = v.x; out[c + 1] = v.y; out[c + 2] = v.z; out[c + 3] = v.w;
        }
    } else if constexpr (Tr::DIST == 2) {
        float2 v = *reinterpret_cast<const float2 *>(best + best_slot<K>(base));
        out[0] = v.x; out[1] = v.y;
    } else {
        out[0] = best[best_slot<K>(base)];
    }
}

// One ACS step: from best_{t-1} (bin) and x_{t-1} to best_t (bout), returning the lane's packed back-pointers
// (bit i·k of the word holds the chosen h of r = lane·RL + i).
template <int K>
__device__ __forceinline__ unsigned long long acs_step(const float *__restrict__ bin, float *__restrict__ bout,
                                                       float xp, int lane,
                                                       const float (&cv)[Trellis<K>::NB][Trellis<K>::RL]) {
    using Tr = Trellis<K>;
    constexpr int CH = (Tr::DIST >= 4) ? 4 : Tr::DIST;  // best values per chunk per h
    constexpr int CI = (Tr::DIST >= 4) ? (4 << K) : Tr::RL;  // r values per chunk
    unsigned long long arg = 0ull;
#pragma unroll
    for (int c0 = 0; c0 < Tr::RL; c0 += CI) {
        float bv[Tr::NB][CH];
#pragma unroll
        for (int h = 0; h < Tr::NB; ++h) {
            const int base = h * (Tr::R >> K) + ((lane * Tr::RL + c0) >> K);
            if constexpr (CH == 4) {
                float4 v = *reinterpret_cast<const float4 *>(bin + best_slot<K>(base));
                bv[h][0] = v.x; bv[h][1] = v.y; bv[h][2] = v.z; bv[h][3] = v.w;
            } else if constexpr (CH == 2) {
                float2 v = *reinterpret_cast<const float2 *>(bin + best_slot<K>(base));
                bv[h][0] = v.x; bv[h][1] = v.y;
            } else {
                bv[h][0] = bin[best_slot<K>(base)];
            }
        }
        float nb4[4];
#pragma unroll
        for (int i = 0; i < CI; ++i) {
            const int ii = c0 + i;
            float m = 0.f;
            int a = 0;
#pragma unroll
            for (int h = 0; h < Tr::NB; ++h) {
                const float d = sub_rn(xp, cv[h][ii]);
                const float c = add_rn(bv[h][i >> K], mul_rn(d, d));
                if (h == 0) {
                    m = c;
                } else if (c < m) {
                    m = c;
                    a = h;
                }
            }
            arg |= (unsigned long long)a << (ii * K);
            nb4[i & 3] = m;
            if ((i & 3) == 3) {
                *reinterpret_cast<float4 *>(bout + best_slot<K>(lane * Tr::RL + ii - 3)) =
                    make_float4(nb4[0], nb4[1], nb4[2], nb4[3]);
            }
        }
    }
    return arg;
}

// Initialises best_0: 0 everywhere (free start) or 0 only at r0 = start & (R-1) (fixed start).
template <int K>
__device__ __forceinline__ void init_best(float *best, int lane, bool has_start, int start) {
    using Tr = Trellis<K>;
    const int r0 = start & (Tr::R - 1);
#pragma unroll
    for (int i = 0; i < Tr::RL; i += 4) {
        float4 v;
        const int r = lane * Tr::RL + i;
        v.x = (!has_start || r + 0 == r0) ? 0.f : __int_as_float(0x7f800000);
        v.y = (!has_start || r + 1 == r0) ? 0.f : __int_as_float(0x7f800000);
        v.z = (!has_start || r + 2 == r0) ? 0.f : __int_as_float(0x7f800000);
        v.w = (!has_start || r + 3 == r0) ? 0.f : __int_as_float(0x7f800000);
        *reinterpret_cast<float4 *>(best + best_slot<K>(r)) = v;
    }
}

// The first state of minimum final cost: cost_{T-1}[s] = best[s >> k] + (x - C[s])^2 over all s, smallest s on ties.
template <int K>
__device__ __forceinline__ int final_argmin(const float *__restrict__ best, float xl, int lane,
                                            const float (&cv)[Trellis<K>::NB][Trellis<K>::RL]) {
    using Tr = Trellis<K>;
    float m = __int_as_float(0x7f800000);
    int ms = 0x7fffffff;
#pragma unroll
    for (int h = 0; h < Tr::NB; ++h) {
        float bv[Tr::DIST];
        read_best<K>(best, lane, h, bv);
#pragma unroll
        for (int i = 0; i < Tr::RL; ++i) {
            const float d = sub_rn(xl, cv[h][i]);
            const float c = add_rn(bv[i >> K], mul_rn(d, d));
            const int s = h * Tr::R + lane * Tr::RL + i;
            // states are visited in increasing order, so a strict < keeps the smallest state on ties;
            // the first visit also accepts +inf so every lane holds a valid state
            if (c < m || ms == 0x7fffffff) {
                m = c;
                ms = s;
            }
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float om = __shfl_xor_sync(0xffffffffu, m, off);
        const int os = __shfl_xor_sync(0xffffffffu, ms, off);
        if (om < m || (om == m && os < ms) || (!(om == om) && false)) {
            m = om;
            ms = os;
        } else if (!(m == m) && !(om == om) && os < ms) {  // both NaN: keep the smaller state
            ms = os;
        }
    }
    return ms;
}

// Follows the back-pointers from the final state. Every lane walks the same path (broadcast reads); lane t ends
// holding the state at position t (t < T).
template <int K>
__device__ __forceinline__ int traceback(const unsigned long long *__restrict__ args, int T, int final_state, int lane) {
    using Tr = Trellis<K>;
    int s = final_state;
    int mine = (lane == T - 1) ? s : 0;
    for (int t = T - 1; t > 0; --t) {
        const int r = s >> K;
        const unsigned long long w = args[t * 32 + r / Tr::RL];
        const int h = (int)((w >> ((r % Tr::RL) * K)) & (Tr::NB - 1));
        s = h * Tr::R + r;
        if (lane == t - 1) mine = s;
    }
    return mine;
}

// Decodes one sequence x_0..x_{T-1} held one per lane (lane t holds x_t, T <= 32) and returns lane t's state.
// best0/best1: two R-float shared buffers; args: T x 32 words of shared (or global) memory.
template <int K>
__device__ __forceinline__ int viterbi_window(float xv, int T, bool has_start, int start,
                                             const float (&cv)[Trellis<K>::NB][Trellis<K>::RL], float *best0,
                                             float *best1, unsigned long long *args, int lane) {
    init_best<K>(best0, lane, has_start, start);
    __syncwarp();
    float *bin = best0, *bout = best1;
    for (int t = 1; t < T; ++t) {
        const float xp = __shfl_sync(0xffffffffu, xv, t - 1);
        const unsigned long long a = acs_step<K>(bin, bout, xp, lane, cv);
        args[t * 32 + lane] = a;
        __syncwarp();
        float *tmp = bin;
        bin = bout;
        bout = tmp;
    }
    const float xl = __shfl_sync(0xffffffffu, xv, T - 1);
    const int fs = final_argmin<K>(bin, xl, lane, cv);
    __syncwarp();
    const int st = traceback<K>(args, T, fs, lane);
    __syncwarp();
    return st;
}

}  // namespace lamq
