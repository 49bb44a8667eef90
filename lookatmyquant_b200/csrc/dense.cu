// Dense fp64 linear algebra on the fp64 tensor cores (mma.sync m16n8k16 f64): the GEMM, blocked Cholesky and
// triangular inverse behind the environment factor U and the QEP target.
//
// Reference: opgraph/frame.py:515-522 (`Environment`: dead inputs, damping, U = chol(cholesky_inverse(chol(H)))ᵀ)
// and quantize.py:1330-1335 (`cross_target`: M = I + α·(solve(H + λ·mean(diag H)·I, Dᵀ))ᵀ), both torch.linalg
// (cuSOLVER) in fp64 there. Here:
//   U: with J the order-reversing permutation, J·H·J = L·Lᵀ gives H = (J·L·J)(J·L·J)ᵀ with J·L·J upper triangular,
//      so the upper Cholesky factor of H⁻¹ is U = (J·L·J)⁻¹ = J·L⁻¹·J — one Cholesky and one triangular inverse
//      (2n³/3 multiply-adds) instead of three factorizations; U is the same unique factor.
//   target = W·M = W + α·((W·D)·Lc⁻ᵀ)·Lc⁻¹ with H + λ·mean(diag H)·I = Lc·Lcᵀ (or M formed once when the stage has
//      more rows than inputs).
// GEMM: mma.sync m16n8k16 f64 on three CTA tile shapes — 128 x 128 (8 warps of 64 x 32) for large products,
// 64 x 64 and 32 x 32 (4 warps) for the small ones at the bottom of the recursion, so they still spread over the
// SMs — K in steps of 16 through a 4-stage cp.async ring (rows padded so fragment loads are bank-conflict free); a
// triangular operand clips each tile's K range.
// Cholesky and inverse together, recursively: (L11, X11) = rec(A11), L21 = A21·X11ᵀ, A22 −= L21·L21ᵀ,
// (L22, X22) = rec(A22), X21 = −X22·(L21·X11) — most of the 2n³/3 multiply-adds in large GEMMs, T = L21·X11 on a
// low-priority stream beside the A22 recursion; 128 x 128 leaves are factored and inverted by one CTA in shared
// memory, 16-column panels on fp64 MMAs (diag_block_kernel).
#include <algorithm>
#include <climits>
#include <map>
#include <mutex>
#include <utility>
#include <vector>

#include "lamq_common.cuh"

namespace lamq {

namespace {

constexpr int NB = 128;  // Cholesky panel / diagonal block

// One CTA tile shape of the GEMM: BM x BN, warps in a WM_ x WN_ grid, each warp FI x FJ m16n8 fragments; K in stages
// of BK (a multiple of 16) through an ST-stage cp.async ring. Row strides are ≡ 4 (mod 16) doubles, so fragment loads
// hit every bank pair the minimum number of times.
template <int BM_, int BN_, int WM_, int WN_, int BK_, int ST_>
struct Tiling {
    static constexpr int BM = BM_, BN = BN_, BK = BK_, ST = ST_, kThreads = 32 * WM_ * WN_, kWarpsN = WN_;
    static constexpr int WTM = BM / WM_, WTN = BN / WN_, FI = WTM / 16, FJ = WTN / 8;
    static constexpr int SA = BK + 4;   // A tile row stride
    static constexpr int SBN = BN + 4;  // B tile (k-major, NN) row stride
    static constexpr int SBT = BK + 4;  // B tile (n-major, NT) row stride
    static constexpr int kATile = BM * SA;
    static constexpr int kBTile = BK * SBN > BN * SBT ? BK * SBN : BN * SBT;
    static constexpr size_t kSmem = ST * (size_t)(kATile + kBTile) * sizeof(double);
    static_assert(FI >= 1 && FJ >= 1 && WTM % 16 == 0 && WTN % 8 == 0 && BK % 16 == 0, "tile shape");
    static_assert(kSmem <= 232448, "shared memory");
};
using TileL = Tiling<128, 128, 2, 4, 32, 3>;  // 8 warps of 64 x 32, K stages of 32
using TileM = Tiling<64, 64, 2, 2, 16, 4>;    // 4 warps of 32 x 32
using TileS = Tiling<32, 32, 2, 2, 16, 4>;    // 4 warps of 16 x 16

struct GemmArgs {
    int M, N, K;
    double alpha, beta;
    const double *A;
    int64_t lda;
    const double *B;
    int64_t ldb;
    double *C;
    int64_t ldc;
    int transB;      // 0: C = αA·B + βC (B is K x N); 1: C = αA·Bᵀ + βC (B is N x K)
    int lower_only;  // skip tiles entirely above the diagonal of C
    int a_lower;     // A is lower triangular (A[m][k] = 0 for k > m): the K loop stops at the tile's last row
    int b_lower;     // the stored B is lower triangular: NN skips k < n, NT skips k > n
    int vec;         // A and B rows are 16-byte aligned: copy two doubles per cp.async
};

// D (16 x 8) += A (16 x 16) · B (16 x 8) in fp64: per thread a0..a7 = A[g + 8·(i&1)][t + 4·(i>>1)],
// b0..b3 = B[t + 4·i][g], c0..c3 = D[g + 8·(i>>1)][2t + (i&1)] (g = lane / 4, t = lane % 4).
__device__ __forceinline__ void dmma16816(double (&c)[4], const double (&a)[8], const double (&b)[4]) {
    asm("mma.sync.aligned.m16n8k16.row.col.f64.f64.f64.f64 {%0, %1, %2, %3}, {%4, %5, %6, %7, %8, %9, %10, %11}, "
        "{%12, %13, %14, %15}, {%0, %1, %2, %3};"
        : "+d"(c[0]), "+d"(c[1]), "+d"(c[2]), "+d"(c[3])
        : "d"(a[0]), "d"(a[1]), "d"(a[2]), "d"(a[3]), "d"(a[4]), "d"(a[5]), "d"(a[6]), "d"(a[7]), "d"(b[0]), "d"(b[1]),
          "d"(b[2]), "d"(b[3]));
}

__device__ __forceinline__ void cp8(double *dst, const double *src, bool ok) {
    const unsigned d = (unsigned)__cvta_generic_to_shared(dst);
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(d), "l"(src), "r"(ok ? 8 : 0) : "memory");
}

// Two doubles; `n` (0, 1 or 2) of them read, the rest zero-filled.
__device__ __forceinline__ void cp16(double *dst, const double *src, int n) {
    const unsigned d = (unsigned)__cvta_generic_to_shared(dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(8 * n) : "memory");
}

// A thread's share of the copy of a ROWS x COLS tile (row stride ld in shared memory) whose top-left element is
// (r0, c0) of a row-major source with row stride lds, shifted by k0 along K (rows when k_rows, else columns): element
// pairs by 16-byte cp.async when VEC (both rows 16-byte aligned), single elements otherwise; what lies outside
// Rmax x Cmax is zero-filled. The slot arithmetic uses compile-time tile widths (shifts), so nothing is precomputed.
template <int kThreads, int ROWS, int COLS, bool VEC>
__device__ __forceinline__ void tile_copy(double *dst, int ld, const double *src, int64_t lds, int r0, int c0, int k0,
                                          bool k_rows, int Rmax, int Cmax) {
    constexpr int PER = VEC ? COLS / 2 : COLS;  // copies per row
    constexpr int SLOTS = (ROWS * PER + kThreads - 1) / kThreads;
    if (k_rows) r0 += k0;
    else c0 += k0;
#pragma unroll
    for (int q = 0; q < SLOTS; ++q) {
        const int e = threadIdx.x + q * kThreads;
        if (ROWS * PER % kThreads != 0 && e >= ROWS * PER) break;
        const int r = e / PER, c = (VEC ? 2 : 1) * (e % PER);
        const int gr = r0 + r, gc = c0 + c;
        if (VEC) {
            int nv = (gr < Rmax) ? min(2, Cmax - gc) : 0;
            nv = nv < 0 ? 0 : nv;
            cp16(dst + r * ld + c, src + (nv > 0 ? (int64_t)gr * lds + gc : 0), nv);
        } else {
            const bool ok = gr < Rmax && gc < Cmax;
            cp8(dst + r * ld + c, src + (ok ? (int64_t)gr * lds + gc : 0), ok);
        }
    }
}

// C = α·A·B(ᵀ) + β·C on the fp64 tensor cores: one T::BM x T::BN tile per CTA, each warp FI x FJ fragments of
// mma.sync m16n8k16 f64 (on B200 the large fp64 shape sustains ~37 TFLOP/s where m8n8k4 with changing operands
// stops near 32), K in steps of 16 through a 4-stage cp.async ring.
template <class T>
__global__ void __launch_bounds__(T::kThreads) dgemm_kernel(GemmArgs g) {
    constexpr int GM = T::BM, GN = T::BN, GK = T::BK, FI = T::FI, FJ = T::FJ, WTM = T::WTM, WTN = T::WTN;
    constexpr int SA = T::SA, SBN = T::SBN, SBT = T::SBT, ST = T::ST;
    constexpr int kATile = T::kATile, kBTile = T::kBTile;
    extern __shared__ __align__(16) double gsm[];
    // Tiles in launch order, the longest K ranges first when an operand is triangular (CTAs start in block order, so
    // the short tiles fill the last wave): A lower — K grows with the row tile; B lower — with the column tile (NT) or
    // shrinks with it (NN).
    int mt = blockIdx.y, nt = blockIdx.x;
    {
        const int lin = blockIdx.x + gridDim.x * blockIdx.y;
        if (g.a_lower) {
            mt = gridDim.y - 1 - lin / gridDim.x;
            nt = lin % gridDim.x;
        } else if (g.b_lower) {
            nt = g.transB ? gridDim.x - 1 - lin / gridDim.y : lin / gridDim.y;
            mt = lin % gridDim.y;
        }
    }
    const int m0 = mt * GM, n0 = nt * GN;
    if (g.lower_only && m0 + GM - 1 < n0) return;  // every row of the tile is above the diagonal
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int wm = (warp / T::kWarpsN) * WTM, wn = (warp % T::kWarpsN) * WTN;  // warp tile WTM x WTN
    const int fg = lane >> 2, ft = lane & 3;
    double acc[FI][FJ][4];
#pragma unroll
    for (int i = 0; i < FI; ++i)
#pragma unroll
        for (int j = 0; j < FJ; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[i][j][e] = 0.0;
    // the K range that can hold non-zero products for this tile
    int kb = 0, ke = g.K;
    if (g.a_lower) ke = min(ke, m0 + GM);
    if (g.b_lower) {
        if (g.transB) ke = min(ke, n0 + GN);
        else kb = max(kb, (n0 / GK) * GK);
    }
    const int ksteps = ke > kb ? (ke - kb + GK - 1) / GK : 0;
    auto As = [&](int s) { return gsm + (size_t)s * (kATile + kBTile); };
    auto Bs = [&](int s) { return gsm + (size_t)s * (kATile + kBTile) + kATile; };
    const bool vec = g.vec != 0;
    constexpr int TH = T::kThreads;
    auto load = [&](int s, int k0) {
        if (vec) {
            tile_copy<TH, GM, GK, true>(As(s), SA, g.A, g.lda, m0, 0, k0, false, g.M, g.K);  // A: GM x GK at (m0, k)
            if (!g.transB) tile_copy<TH, GK, GN, true>(Bs(s), SBN, g.B, g.ldb, 0, n0, k0, true, g.K, g.N);
            else tile_copy<TH, GN, GK, true>(Bs(s), SBT, g.B, g.ldb, n0, 0, k0, false, g.N, g.K);
        } else {
            tile_copy<TH, GM, GK, false>(As(s), SA, g.A, g.lda, m0, 0, k0, false, g.M, g.K);
            if (!g.transB) tile_copy<TH, GK, GN, false>(Bs(s), SBN, g.B, g.ldb, 0, n0, k0, true, g.K, g.N);
            else tile_copy<TH, GN, GK, false>(Bs(s), SBT, g.B, g.ldb, n0, 0, k0, false, g.N, g.K);
        }
    };
#pragma unroll
    for (int s = 0; s < ST - 1; ++s) {
        if (s < ksteps) load(s, kb + s * GK);
        asm volatile("cp.async.commit_group;" ::: "memory");
    }
    for (int ks = 0; ks < ksteps; ++ks) {
        asm volatile("cp.async.wait_group %0;" ::"n"(ST - 2) : "memory");
        __syncthreads();  // stage ks is in, and stage ks − 1 is free for the next load
        const int nxt = ks + ST - 1;
        if (nxt < ksteps) load(nxt % ST, kb + nxt * GK);
        asm volatile("cp.async.commit_group;" ::: "memory");
        const double *A = As(ks % ST), *B = Bs(ks % ST);
#pragma unroll
        for (int kk = 0; kk < GK; kk += 16) {
            double bf[FJ][4];
#pragma unroll
            for (int j = 0; j < FJ; ++j)
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    bf[j][e] = g.transB ? B[(wn + 8 * j + fg) * SBT + kk + ft + 4 * e]
                                        : B[(kk + ft + 4 * e) * SBN + wn + 8 * j + fg];
#pragma unroll
            for (int i = 0; i < FI; ++i) {
                double af[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) af[e] = A[(wm + 16 * i + fg + 8 * (e & 1)) * SA + kk + ft + 4 * (e >> 1)];
#pragma unroll
                for (int j = 0; j < FJ; ++j) dmma16816(acc[i][j], af, bf[j]);
            }
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    // D fragment: rows g and g + 8 of each 16 x 8 block, columns 2t, 2t + 1
#pragma unroll
    for (int i = 0; i < FI; ++i) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int r = m0 + wm + 16 * i + fg + 8 * h;
            if (r >= g.M) continue;
#pragma unroll
            for (int j = 0; j < FJ; ++j) {
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int c = n0 + wn + 8 * j + 2 * ft + e;
                    if (c >= g.N) continue;
                    double *p = g.C + (int64_t)r * g.ldc + c;
                    const double v = g.alpha * acc[i][j][2 * h + e];
                    *p = (g.beta == 0.0) ? v : fma(g.beta, *p, v);
                }
            }
        }
    }
}

// Cholesky and inverse of a 16 x 16 block by one warp: S (row stride ld) holds the block's lower part on entry and L
// (strict upper zero) on return; Xd (row stride kLeafLdd) receives L⁻¹ (strict upper zero). Lane r (and r + 16, which
// repeats it) holds row r; column k: r_k = rsqrt(a_kk) from lane k, l = a[k]·r_k, a[c] −= l·l_c (l_c shuffled from
// lane c). Entries above the diagonal take updates that are never read and are stored as zero. Column r of the inverse
// is then formed by lane r, right-looking: x_m = acc_m·r_m, acc_q −= L[q][m]·x_m (q > m), acc starting at e_r.
constexpr int kLeafLdd = 20;  // ≡ 4 (mod 16) doubles: fragment loads hit each bank pair twice, the minimum

__device__ __forceinline__ void chol_inv16(double *S, int ld, double *Xd, int *bad) {
    const int lane = threadIdx.x & 31, r = lane & 15;
    double a[16], rinv[16];
#pragma unroll
    for (int c = 0; c < 16; ++c) a[c] = S[r * ld + c];
#pragma unroll
    for (int k = 0; k < 16; ++k) {
        const double d = __shfl_sync(0xffffffffu, a[k], k);
        if (lane == 0 && !(d > 0.0)) *bad = 1;
        rinv[k] = rsqrt(d);
        const double l = a[k] * rinv[k];
        a[k] = l;
#pragma unroll
        for (int c = k + 1; c < 16; ++c) a[c] = fma(-l, __shfl_sync(0xffffffffu, l, c), a[c]);
    }
    if (lane < 16) {
#pragma unroll
        for (int c = 0; c < 16; ++c) S[r * ld + c] = (c <= r) ? a[c] : 0.0;
    }
    __syncwarp();
    double acc[16];
#pragma unroll
    for (int m = 0; m < 16; ++m) acc[m] = (m == r) ? 1.0 : 0.0;
#pragma unroll
    for (int m = 0; m < 16; ++m) {
        const double x = acc[m] * rinv[m];
        acc[m] = x;
#pragma unroll
        for (int q = m + 1; q < 16; ++q) acc[q] = fma(-S[q * ld + m], x, acc[q]);
    }
    if (lane < 16) {
#pragma unroll
        for (int m = 0; m < 16; ++m) Xd[m * kLeafLdd + r] = acc[m];  // X[m][r]: zero for m < r
    }
    __syncwarp();
}

// Factors the nb x nb diagonal block at A[k0][k0] in place (lower Cholesky; the block's strict upper part set to zero)
// and writes its inverse to X[k0][k0] (lower, strict upper zero). A non-positive pivot sets *status = LAMQ_ERR_NOT_PD.
// Blocked by 16-column panels on the fp64 tensor cores, 8 warps, warp w owning rows [16w, 16w + 16); the block is
// padded to a multiple of 16 with the identity and kept in shared memory (row stride ≡ 4 mod 16 doubles). The rows of
// the inverse, R (warp w: its rows, 16 column tiles of 16 x 8 in registers, starting at I), are formed in the same
// panel loop: X[q] = X_qq·R[q] once R[q] has taken every R[q] −= L[q][j]·X[j], j < q. Panel p:
//   (a) warp p factors and inverts its diagonal 16 x 16 block (L_pp, X_pp = L_pp⁻¹);                     | barrier |
//   (b) every later warp forms its rows of the panel, L21 = A21·X_ppᵀ (two m16n8k16 MMAs), and stores them; warp p + 1
//       then updates its diagonal block (the next panel's) from its own rows; warp p stores L_pp;         | barrier |
//   (c) warps w > p + 1 update their trailing tiles up to their own diagonal block, A22 −= L21·L21ᵀ, and take
//       R[w] −= L[w][p−1]·X[p−1]; warp p takes its last two updates (with X[p−2] and X[p−1]) and forms X[p] = X_pp·R[p]
//       into one of two row-panel buffers (and global memory); warp p + 1 goes on to factor.
// The chain that sets the leaf's time is (a) → (b) → (a) of the next panel: every product of (c), the inverse's
// included, runs beside the next factor step, and warp p + 1 defers its update with X[p − 1] to the panel it factors.
constexpr int kLeafThreads = 256;
constexpr int kLeafLd = NB + 4;
constexpr size_t kLeafSmem = (size_t)(NB * kLeafLd + 8 * 16 * kLeafLdd + 2 * 16 * kLeafLd) * sizeof(double);

// R[w] −= L[w][q]·X[q] over the column tiles ct < 2q + 2 (the only non-zero ones of X[q]): Lq = this warp's band at
// column 16q, Xq = the row panel of X[q].
__device__ __forceinline__ void leaf_inverse_update(double (&R)[16][4], const double *Lq, const double *Xq, int q,
                                                    int g, int tq) {
    double af[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) af[e] = -Lq[(g + 8 * (e & 1)) * kLeafLd + tq + 4 * (e >> 1)];
#pragma unroll
    for (int ct = 0; ct < 16; ++ct) {
        if (ct >= 2 * q + 2) continue;  // warp-uniform
        double bf[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) bf[e] = Xq[(tq + 4 * e) * kLeafLd + 8 * ct + g];
        dmma16816(R[ct], af, bf);
    }
}

// This warp's band −= L21·L21ᵀ over its column tiles ct0 .. ct1 (L21: the band's and the tiles' rows at column j0).
__device__ __forceinline__ void leaf_trailing(double *band, const double *Ls, int j0, int ct0, int ct1, int g,
                                              int tq) {
    double af[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) af[e] = -band[(g + 8 * (e & 1)) * kLeafLd + j0 + tq + 4 * (e >> 1)];
#pragma unroll
    for (int ct = 2; ct < 16; ++ct) {  // unrolled so the independent tiles' MMAs overlap
        if (ct < ct0 || ct > ct1) continue;  // warp-uniform
        double bf[4], cf[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) bf[e] = Ls[(8 * ct + g) * kLeafLd + j0 + tq + 4 * e];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const double2 v = *reinterpret_cast<const double2 *>(band + (g + 8 * h) * kLeafLd + 8 * ct + 2 * tq);
            cf[2 * h] = v.x;
            cf[2 * h + 1] = v.y;
        }
        dmma16816(cf, af, bf);
#pragma unroll
        for (int h = 0; h < 2; ++h)
            *reinterpret_cast<double2 *>(band + (g + 8 * h) * kLeafLd + 8 * ct + 2 * tq) =
                make_double2(cf[2 * h], cf[2 * h + 1]);
    }
}

__global__ void __launch_bounds__(kLeafThreads, 1) diag_block_kernel(double *A, int64_t lda, int k0, int nb,
                                                                     double *X, int64_t ldx, int *status) {
    extern __shared__ __align__(16) double lsm[];
    double *Ls = lsm;                         // the padded block, row-major; L on the way out
    double *Xd = Ls + NB * kLeafLd;           // the diagonal blocks' inverses, 16 x kLeafLdd each
    double *Xp0 = Xd + 8 * 16 * kLeafLdd;     // two row panels of L⁻¹: X[q] in Xp0 + (q & 1)·16·kLeafLd
    __shared__ int bad;
    const int t = threadIdx.x, w = t >> 5, lane = t & 31, g = lane >> 2, tq = lane & 3;
    const int P = (nb + 15) >> 4, nbp = 16 * P;
    double *Ab = A + (int64_t)k0 * lda + k0;
    // staging: thread t covers columns 2(t % 64), 2(t % 64) + 1 of rows t / 64, t / 64 + 4, …: 32 loads in flight
    // (16-byte loads when the rows allow them); the strict upper part is not read and is zeroed in global memory here
    {
        const int c = 2 * (t & 63), i0 = t >> 6;
        const bool vec = (lda & 1) == 0 && (reinterpret_cast<uintptr_t>(Ab) & 15) == 0;
        double v0[32], v1[32];
#pragma unroll
        for (int u = 0; u < 32; ++u) {
            const int i = i0 + 4 * u;
            const double *src = Ab + (int64_t)i * lda + c;
            if (vec && i < nb && c + 1 < nb && c + 1 <= i) {
                const double2 v = __ldg(reinterpret_cast<const double2 *>(src));
                v0[u] = v.x;
                v1[u] = v.y;
            } else {
                v0[u] = (i < nb && c < nb && c <= i) ? __ldg(src) : 0.0;
                v1[u] = (i < nb && c + 1 < nb && c + 1 <= i) ? __ldg(src + 1) : 0.0;
            }
        }
#pragma unroll
        for (int u = 0; u < 32; ++u) {
            const int i = i0 + 4 * u;
            if (i < nbp && c < nbp)
                *reinterpret_cast<double2 *>(Ls + i * kLeafLd + c) =
                    make_double2((i < nb && c < nb) ? v0[u] : (i == c ? 1.0 : 0.0),
                                 (i < nb && c + 1 < nb) ? v1[u] : (i == c + 1 ? 1.0 : 0.0));
            if (i < nb && c < nb && c > i) Ab[(int64_t)i * lda + c] = 0.0;
            if (i < nb && c + 1 < nb && c + 1 > i) Ab[(int64_t)i * lda + c + 1] = 0.0;
        }
    }
    if (t == 0) bad = 0;
    double R[16][4];
#pragma unroll
    for (int ct = 0; ct < 16; ++ct)
#pragma unroll
        for (int e = 0; e < 4; ++e) R[ct][e] = (16 * w + g + 8 * (e >> 1) == 8 * ct + 2 * tq + (e & 1)) ? 1.0 : 0.0;
    __syncthreads();
    double *band = Ls + (16 * w) * kLeafLd;
    for (int p = 0; p < P; ++p) {
        const int j0 = 16 * p;
        // (a)
        if (w == p) chol_inv16(Ls + j0 * kLeafLd + j0, kLeafLd, Xd + p * 16 * kLeafLdd, &bad);
        __syncthreads();
        // (b)
        const bool later = w > p && w < P;
        if (later) {  // L21 = A21 · X_ppᵀ for rows [16w, 16w + 16), into shared memory and global memory
            double af[8], b0[4], b1[4], d0[4] = {0.0, 0.0, 0.0, 0.0}, d1[4] = {0.0, 0.0, 0.0, 0.0};
            const double *xp = Xd + p * 16 * kLeafLdd;
#pragma unroll
            for (int e = 0; e < 8; ++e) af[e] = band[(g + 8 * (e & 1)) * kLeafLd + j0 + tq + 4 * (e >> 1)];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                b0[e] = xp[g * kLeafLdd + tq + 4 * e];
                b1[e] = xp[(8 + g) * kLeafLdd + tq + 4 * e];
            }
            dmma16816(d0, af, b0);
            dmma16816(d1, af, b1);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int i = 16 * w + g + 8 * h, c = j0 + 2 * tq;
                double *row = band + (g + 8 * h) * kLeafLd + c;
                *reinterpret_cast<double2 *>(row) = make_double2(d0[2 * h], d0[2 * h + 1]);
                *reinterpret_cast<double2 *>(row + 8) = make_double2(d1[2 * h], d1[2 * h + 1]);
                if (i < nb) {
                    double *dst = Ab + (int64_t)i * lda + c;
                    if (c < nb) dst[0] = d0[2 * h];
                    if (c + 1 < nb) dst[1] = d0[2 * h + 1];
                    if (c + 8 < nb) dst[8] = d1[2 * h];
                    if (c + 9 < nb) dst[9] = d1[2 * h + 1];
                }
            }
            if (w == p + 1) {  // the next panel's diagonal block, from this warp's own rows: A_dd −= L21·L21ᵀ
                __syncwarp();
                leaf_trailing(band, Ls, j0, 2 * w, 2 * w + 1, g, tq);
            }
        } else if (w == p) {  // L_pp to global memory
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const int r = (lane >> 4) + 2 * e, c = lane & 15, i = j0 + r;
                if (i < nb && j0 + c < nb) Ab[(int64_t)i * lda + j0 + c] = Ls[i * kLeafLd + j0 + c];
            }
        }
        __syncthreads();
        // (c)
        if (later && w > p + 1) {  // A22 −= L21 · L21ᵀ over this band's column tiles 2p + 2 .. 2w + 1
            leaf_trailing(band, Ls, j0, 2 * p + 2, 2 * w + 1, g, tq);
            if (p >= 1) leaf_inverse_update(R, band + 16 * (p - 1), Xp0 + ((p - 1) & 1) * 16 * kLeafLd, p - 1, g, tq);
        } else if (w == p) {  // the last updates of R[p], then X[p] = X_pp · R[p]
            if (p >= 2) leaf_inverse_update(R, band + 16 * (p - 2), Xp0 + (p & 1) * 16 * kLeafLd, p - 2, g, tq);
            if (p >= 1) leaf_inverse_update(R, band + 16 * (p - 1), Xp0 + ((p - 1) & 1) * 16 * kLeafLd, p - 1, g, tq);
            double *Xp = Xp0 + (p & 1) * 16 * kLeafLd;  // X[p − 2]'s buffer, read above by this warp only
            __syncwarp();
#pragma unroll
            for (int ct = 0; ct < 16; ++ct) {
                if (ct >= 2 * p + 2) continue;
#pragma unroll
                for (int h = 0; h < 2; ++h)
                    *reinterpret_cast<double2 *>(Xp + (g + 8 * h) * kLeafLd + 8 * ct + 2 * tq) =
                        make_double2(R[ct][2 * h], R[ct][2 * h + 1]);
            }
            __syncwarp();
            double af[8];
            const double *xq = Xd + p * 16 * kLeafLdd;
#pragma unroll
            for (int e = 0; e < 8; ++e) af[e] = xq[(g + 8 * (e & 1)) * kLeafLdd + tq + 4 * (e >> 1)];
#pragma unroll
            for (int ct = 0; ct < 16; ++ct) {
                if (ct >= 2 * p + 2) continue;
                double bf[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) bf[e] = Xp[(tq + 4 * e) * kLeafLd + 8 * ct + g];
#pragma unroll
                for (int e = 0; e < 4; ++e) R[ct][e] = 0.0;
                dmma16816(R[ct], af, bf);
            }
            __syncwarp();
#pragma unroll
            for (int ct = 0; ct < 16; ++ct) {
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int i = j0 + g + 8 * h, c = 8 * ct + 2 * tq;
                    const double v0 = (ct < 2 * p + 2) ? R[ct][2 * h] : 0.0;
                    const double v1 = (ct < 2 * p + 2) ? R[ct][2 * h + 1] : 0.0;
                    if (ct < 2 * p + 2)
                        *reinterpret_cast<double2 *>(Xp + (g + 8 * h) * kLeafLd + c) = make_double2(v0, v1);
                    if (i < nb) {
                        double *xr = X + (int64_t)(k0 + i) * ldx + k0;
                        if (c < nb) xr[c] = v0;
                        if (c + 1 < nb) xr[c + 1] = v1;
                    }
                }
            }
        }
    }
    __syncthreads();
    if (t == 0 && bad) atomicCAS(status, 0, LAMQ_ERR_NOT_PD);
}

// dst[r][c] = src[r][c] for an rows x cols block
__global__ void copy_block_kernel(const double *src, int64_t lds, double *dst, int64_t ldd, int rows, int cols) {
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < (int64_t)rows * cols;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int r = (int)(e / cols), c = (int)(e % cols);
        dst[(int64_t)r * ldd + c] = src[(int64_t)r * lds + c];
    }
}

// The n x n identity.
__global__ void identity_kernel(double *A, int64_t lda, int n) {
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < (int64_t)n * n;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int r = (int)(e / n), c = (int)(e % n);
        A[(int64_t)r * lda + c] = (r == c) ? 1.0 : 0.0;
    }
}

// Zero the strict upper triangle of an n x n matrix.
__global__ void zero_upper_kernel(double *A, int64_t lda, int n) {
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < (int64_t)n * n;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int r = (int)(e / n), c = (int)(e % n);
        if (c > r) A[(int64_t)r * lda + c] = 0.0;
    }
}

// out[i][j] = in[n-1-i][n-1-j]
__global__ void flip_kernel(const double *in, int64_t ldi, double *out, int64_t ldo, int n) {
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < (int64_t)n * n;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int r = (int)(e / n), c = (int)(e % n);
        out[(int64_t)r * ldo + c] = in[(int64_t)(n - 1 - r) * ldi + (n - 1 - c)];
    }
}

// Environment preparation (frame.py:517-521): dead[i] = (H[i][i] == 0); those diagonals become 1; then
// H += damp · mean(diag H) · I. One CTA; n <= 65536.
__global__ void env_prep_kernel(double *H, int64_t ldh, int n, double damp, uint8_t *dead) {
    __shared__ double part[1024];
    double s = 0.0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        double d = H[(int64_t)i * ldh + i];
        const bool z = (d == 0.0);
        if (dead) dead[i] = z ? 1 : 0;
        if (z) {
            d = 1.0;
            H[(int64_t)i * ldh + i] = 1.0;
        }
        s += d;
    }
    part[threadIdx.x] = s;
    __syncthreads();
    for (int w = blockDim.x / 2; w > 0; w >>= 1) {
        if (threadIdx.x < w) part[threadIdx.x] += part[threadIdx.x + w];
        __syncthreads();
    }
    const double add = damp * (part[0] / n);
    for (int i = threadIdx.x; i < n; i += blockDim.x) H[(int64_t)i * ldh + i] += add;
}

// A += lam · mean(diag A) · I (the diagonal only; one CTA)
__global__ void ridge_diag_kernel(double *A, int64_t lda, int n, double lam) {
    __shared__ double part[1024];
    double s = 0.0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) s += A[(int64_t)i * lda + i];
    part[threadIdx.x] = s;
    __syncthreads();
    for (int w = blockDim.x / 2; w > 0; w >>= 1) {
        if (threadIdx.x < w) part[threadIdx.x] += part[threadIdx.x + w];
        __syncthreads();
    }
    const double add = lam * (part[0] / n);
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) A[(int64_t)i * lda + i] += add;
}

// E = A − B (B may be null: E = A), rows x n, into a dense buffer.
__global__ void diff_kernel(const double *A, int64_t lda, const double *B, int64_t ldb, double *E, int rows, int n) {
    const int64_t total = (int64_t)rows * n;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = e / n, j = e % n;
        E[e] = B ? A[r * lda + j] - B[r * ldb + j] : A[r * lda + j];
    }
}

// loss[r] = Σ_j P[r][j]·E[r][j] (P = E·H): one warp per row, lanes strided over j, then a fixed shuffle tree.
__global__ void row_dot_kernel(const double *P, const double *E, int rows, int n, double *loss) {
    const int warp = (int)((blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
    if (warp >= rows) return;
    const double *p = P + (int64_t)warp * n, *e = E + (int64_t)warp * n;
    double acc = 0.0;
    for (int j = lane; j < n; j += 32) acc = fma(p[j], e[j], acc);
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_down_sync(0xffffffffu, acc, o);
    if (lane == 0) loss[warp] = acc;
}

// total = Σ_r loss[r] in a fixed order (one CTA: strided partial sums, then a tree), so repeated calls agree bit
// for bit.
__global__ void sum_rows_kernel(const double *loss, int64_t rows, double *total) {
    __shared__ double red[256];
    double acc = 0.0;
    for (int64_t r = threadIdx.x; r < rows; r += blockDim.x) acc += loss[r];
    red[threadIdx.x] = acc;
    __syncthreads();
    for (int h = blockDim.x / 2; h > 0; h >>= 1) {
        if ((int)threadIdx.x < h) red[threadIdx.x] += red[threadIdx.x + h];
        __syncthreads();
    }
    if (threadIdx.x == 0) *total = red[0];
}

constexpr int kProxyRowBlock = 4096;  // rows per E·H product (bounds the workspace)

int grid_for(int64_t n) { return (int)std::min<int64_t>((n + 255) / 256, 148 * 16); }

template <class T>
int launch_dgemm(cudaStream_t s, const GemmArgs &g) {
    const cudaError_t e = smem_limit_once((const void *)dgemm_kernel<T>, (int)T::kSmem);
    if (e != cudaSuccess) {
        set_error("dgemm: %s", cudaGetErrorString(e));
        return LAMQ_ERR_CUDA;
    }
    dim3 grid((g.N + T::BN - 1) / T::BN, (g.M + T::BM - 1) / T::BM);
    dgemm_kernel<T><<<grid, T::kThreads, T::kSmem, s>>>(g);
    LAMQ_CHECK_LAUNCH("dgemm");
    return LAMQ_OK;
}

// CTA tiles of a b x b tiling of an M x N product (half of them when only the lower triangle is computed).
int64_t tile_count(int M, int N, int b, int lower_only) {
    const int64_t t = (int64_t)((M + b - 1) / b) * ((N + b - 1) / b);
    return lower_only ? (t + (M + b - 1) / b) / 2 : t;
}

// The tile shape: the largest whose grid still fills most of the 148 SMs (smaller tiles re-read more of A and B
// from L2, which only matters for products large enough to use the 128 x 128 tiles anyway).
int dgemm(cudaStream_t s, int transB, int M, int N, int K, double alpha, const double *A, int64_t lda,
          const double *B, int64_t ldb, double beta, double *C, int64_t ldc, int lower_only = 0, int a_lower = 0,
          int b_lower = 0) {
    if (M <= 0 || N <= 0) return LAMQ_OK;
    const bool vec = ((uintptr_t)A % 16 == 0) && (lda % 2 == 0) && ((uintptr_t)B % 16 == 0) && (ldb % 2 == 0);
    GemmArgs g{M, N, K, alpha, beta, A, lda, B, ldb, C, ldc, transB, lower_only, a_lower, b_lower, vec ? 1 : 0};
    constexpr int64_t kFill = 120;
    if (tile_count(M, N, 128, lower_only) >= kFill) return launch_dgemm<TileL>(s, g);
    if (tile_count(M, N, 64, lower_only) >= kFill) return launch_dgemm<TileM>(s, g);
    return launch_dgemm<TileS>(s, g);
}

// Recursive Cholesky with inverse of the block [o, o+m) of A (lower part read); L⁻¹ goes to X's lower part, and A
// (scratch) keeps only the factor's diagonal blocks. [[A11, ·], [A21, A22]]: (L11, X11) = rec(A11); L21 = A21·X11ᵀ
// (held in X21's place); A22 −= L21·L21ᵀ; (L22, X22) = rec(A22); X21 = −X22·(L21·X11).
// The recursion's chain runs on a high-priority stream; T = L21·X11 depends only on L21 and X11, so it runs on a
// low-priority stream of its depth while A22 is updated and factored (whose leaves and small products leave most SMs
// idle), and is joined before X21. T of depth d goes to its own buffer W_d.
constexpr int kAuxStreams = 8;
constexpr int kMaxDepth = 32;

struct FactorStreams {
    cudaStream_t crit = nullptr;
    cudaStream_t aux[kAuxStreams] = {};
};

// One set of internal streams per (device, caller stream): calls made on different streams keep running side by side.
// At most kMaxStreamSets sets per device are created; callers beyond them share the existing sets in turn (still
// correct — every call forks from its caller's stream and joins back — only no longer side by side).
constexpr int kMaxStreamSets = 8;

int factor_streams(cudaStream_t caller, FactorStreams **out) {
    static std::mutex mu;
    static std::map<std::pair<int, cudaStream_t>, FactorStreams *> assigned;
    static std::map<int, std::vector<FactorStreams *>> sets;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        set_error("factorization: %s", cudaGetErrorString(e));
        return LAMQ_ERR_CUDA;
    }
    std::lock_guard<std::mutex> lock(mu);
    auto it = assigned.find({dev, caller});
    if (it == assigned.end()) {
        std::vector<FactorStreams *> &mine = sets[dev];
        FactorStreams *fs = nullptr;
        if ((int)mine.size() < kMaxStreamSets) {
            int least = 0, greatest = 0;
            FactorStreams made;
            e = cudaDeviceGetStreamPriorityRange(&least, &greatest);
            if (e == cudaSuccess) e = cudaStreamCreateWithPriority(&made.crit, cudaStreamNonBlocking, greatest);
            for (int d = 0; e == cudaSuccess && d < kAuxStreams; ++d)
                e = cudaStreamCreateWithPriority(&made.aux[d], cudaStreamNonBlocking, least);
            if (e != cudaSuccess) {
                set_error("factorization streams: %s", cudaGetErrorString(e));
                return LAMQ_ERR_CUDA;
            }
            fs = new FactorStreams(made);  // kept for the life of the process, like the streams themselves
            mine.push_back(fs);
        } else {
            fs = mine[assigned.size() % mine.size()];
        }
        it = assigned.emplace(std::make_pair(dev, caller), fs).first;
    }
    *out = it->second;
    return LAMQ_OK;
}

struct FactorCtx {
    FactorStreams *fs;
    cudaEvent_t fork;
    cudaEvent_t join[kMaxDepth];
    double *W[kMaxDepth];  // T buffers per depth
    int *status;
};

// The largest T (m2 x m1 doubles) at each depth of the recursion over m.
void t_sizes(int m, int d, std::vector<size_t> &mx) {
    if (m <= NB) return;
    const int nblk = (m + NB - 1) / NB;
    const int m1 = (nblk / 2) * NB, m2 = m - m1;
    if ((int)mx.size() <= d) mx.resize(d + 1, 0);
    mx[d] = std::max(mx[d], (size_t)m2 * m1);
    t_sizes(m1, d + 1, mx);
    t_sizes(m2, d + 1, mx);
}

size_t w_elems(int n) {
    std::vector<size_t> mx;
    t_sizes(n, 0, mx);
    size_t total = 0;
    for (size_t v : mx) total += (v + 31) / 32 * 32;  // 256-byte aligned buffers
    return total;
}

int chol_inv_rec(FactorCtx &c, double *A, int64_t lda, double *X, int64_t ldx, int o, int m, int depth) {
    cudaStream_t s = c.fs->crit;
    if (m <= NB) {
        diag_block_kernel<<<1, kLeafThreads, kLeafSmem, s>>>(A, lda, o, m, X, ldx, c.status);
        LAMQ_CHECK_LAUNCH("diagonal block");
        return LAMQ_OK;
    }
    if (depth >= kMaxDepth) {
        set_error("factorization: recursion deeper than %d", kMaxDepth);
        return LAMQ_ERR_INVALID;
    }
    const int nblk = (m + NB - 1) / NB;
    const int m1 = (nblk / 2) * NB, m2 = m - m1;
    int st = chol_inv_rec(c, A, lda, X, ldx, o, m1, depth + 1);
    if (st) return st;
    const double *A21 = A + (int64_t)(o + m1) * lda + o;
    double *A22 = A + (int64_t)(o + m1) * lda + o + m1;
    const double *X11 = X + (int64_t)o * ldx + o;
    double *X21 = X + (int64_t)(o + m1) * ldx + o;
    const double *X22 = X + (int64_t)(o + m1) * ldx + o + m1;
    double *T = c.W[depth];
    // L21 = A21·X11ᵀ (X11 lower), held in X21's place until X21 is formed
    st = dgemm(s, 1, m2, m1, m1, 1.0, A21, lda, X11, ldx, 0.0, X21, ldx, 0, 0, 1);
    if (st) return st;
    // T = L21·X11 beside the rest of this node
    cudaStream_t aux = c.fs->aux[std::min(depth, kAuxStreams - 1)];
    cudaError_t e = cudaEventRecord(c.fork, s);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(aux, c.fork, 0);
    if (e != cudaSuccess) {
        set_error("factorization fork: %s", cudaGetErrorString(e));
        return LAMQ_ERR_CUDA;
    }
    st = dgemm(aux, 0, m2, m1, m1, 1.0, X21, ldx, X11, ldx, 0.0, T, m1, 0, 0, 1);
    if (st) return st;
    e = cudaEventRecord(c.join[depth], aux);
    if (e != cudaSuccess) {
        set_error("factorization join: %s", cudaGetErrorString(e));
        return LAMQ_ERR_CUDA;
    }
    // A22 -= L21·L21ᵀ (lower part)
    st = dgemm(s, 1, m2, m2, m1, -1.0, X21, ldx, X21, ldx, 1.0, A22, lda, 1);
    if (st) return st;
    st = chol_inv_rec(c, A, lda, X, ldx, o + m1, m2, depth + 1);
    if (st) return st;
    e = cudaStreamWaitEvent(s, c.join[depth], 0);
    if (e != cudaSuccess) {
        set_error("factorization join: %s", cudaGetErrorString(e));
        return LAMQ_ERR_CUDA;
    }
    // X21 = −X22·T: X22 lower triangular
    return dgemm(s, 0, m2, m1, m2, -1.0, X22, ldx, T, m1, 0.0, X21, ldx, 0, 1, 0);
}

// L⁻¹ of the n x n matrix in A (lower part read; A is scratch) into X's lower part (strict upper zeroed), on
// `caller`'s stream order (internal streams joined before the return).
int chol_inv(cudaStream_t caller, double *A, int64_t lda, double *X, int64_t ldx, int n, double *W, int *status) {
    cudaError_t e = smem_limit_once((const void *)diag_block_kernel, (int)kLeafSmem);
    if (e != cudaSuccess) {
        set_error("cholesky leaf: %s", cudaGetErrorString(e));
        return LAMQ_ERR_CUDA;
    }
    FactorCtx c{};
    int st = factor_streams(caller, &c.fs);
    if (st) return st;
    c.status = status;
    std::vector<size_t> mx;
    t_sizes(n, 0, mx);
    if (mx.size() > (size_t)kMaxDepth) {
        set_error("factorization: n = %d is too large", n);
        return LAMQ_ERR_INVALID;
    }
    for (size_t d = 0; d < mx.size(); ++d) {
        c.W[d] = W;
        W += (mx[d] + 31) / 32 * 32;
    }
    const int depths = (int)mx.size();
    e = cudaEventCreateWithFlags(&c.fork, cudaEventDisableTiming);
    for (int d = 0; e == cudaSuccess && d < depths; ++d) e = cudaEventCreateWithFlags(&c.join[d], cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventRecord(c.fork, caller);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(c.fs->crit, c.fork, 0);
    if (e != cudaSuccess) {
        set_error("factorization: %s", cudaGetErrorString(e));
        return LAMQ_ERR_CUDA;
    }
    st = chol_inv_rec(c, A, lda, X, ldx, 0, n, 0);
    if (st == LAMQ_OK) {
        zero_upper_kernel<<<grid_for((int64_t)n * n), 256, 0, c.fs->crit>>>(X, ldx, n);
        cudaError_t le = cudaGetLastError();
        if (le != cudaSuccess) {
            set_error("zero upper: %s", cudaGetErrorString(le));
            st = LAMQ_ERR_CUDA;
        }
    }
    // the caller's stream continues after the internal streams' work (also on an error, so nothing is left behind)
    e = cudaEventRecord(c.fork, c.fs->crit);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(caller, c.fork, 0);
    cudaEventDestroy(c.fork);
    for (int d = 0; d < depths; ++d)
        if (c.join[d]) cudaEventDestroy(c.join[d]);
    if (st == LAMQ_OK && e != cudaSuccess) {
        set_error("factorization: %s", cudaGetErrorString(e));
        st = LAMQ_ERR_CUDA;
    }
    return st;
}

}  // namespace

}  // namespace lamq

using namespace lamq;

extern "C" int lamq_dgemm(int transB, int M, int N, int K, double alpha, const double *A, int64_t lda,
                          const double *B, int64_t ldb, double beta, double *C, int64_t ldc, lamq_stream_t stream) {
    LAMQ_REQUIRE(M >= 0 && N >= 0 && K >= 0, "lamq_dgemm: negative shape");
    LAMQ_REQUIRE(M == 0 || N == 0 || (A && B && C), "lamq_dgemm: null pointer");
    return dgemm((cudaStream_t)stream, transB, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc);
}

extern "C" size_t lamq_factor_workspace_size(int n) {
    if (n <= 0) return 0;
    return (2 * (size_t)n * n + w_elems(n)) * sizeof(double) + 64;
}

extern "C" int lamq_cholesky_inverse_lower(double *A, int64_t lda, int n, void *workspace, size_t workspace_bytes,
                                           int *status, lamq_stream_t stream) {
    LAMQ_REQUIRE(n >= 0 && lda >= n, "lamq_cholesky_inverse_lower: bad shape");
    if (n == 0) return LAMQ_OK;
    LAMQ_REQUIRE(A && workspace && status, "lamq_cholesky_inverse_lower: null pointer");
    LAMQ_REQUIRE(workspace_bytes >= lamq_factor_workspace_size(n), "lamq_cholesky_inverse_lower: workspace too small");
    cudaStream_t s = (cudaStream_t)stream;
    double *L = reinterpret_cast<double *>(workspace);  // the factor (scratch)
    double *W = L + (size_t)n * n;
    copy_block_kernel<<<grid_for((int64_t)n * n), 256, 0, s>>>(A, lda, L, n, n, n);
    LAMQ_CHECK_LAUNCH("lamq_cholesky_inverse_lower copy");
    return chol_inv(s, L, n, A, lda, n, W, status);
}

extern "C" int lamq_env_factor(const double *H, int64_t ldh, int n, double damp, double *U, int64_t ldu,
                               uint8_t *dead, void *workspace, size_t workspace_bytes, int *status,
                               lamq_stream_t stream) {
    LAMQ_REQUIRE(n >= 0 && ldh >= n && ldu >= n, "lamq_env_factor: bad shape");
    if (n == 0) return LAMQ_OK;
    LAMQ_REQUIRE(H && U && workspace && status && H != U, "lamq_env_factor: null or aliased pointer");
    LAMQ_REQUIRE(workspace_bytes >= lamq_factor_workspace_size(n), "lamq_env_factor: workspace too small");
    cudaStream_t s = (cudaStream_t)stream;
    double *F = reinterpret_cast<double *>(workspace);  // flipped damped H, then its Cholesky factor
    double *X = F + (size_t)n * n;                      // the factor's inverse
    double *W = X + (size_t)n * n;
    copy_block_kernel<<<grid_for((int64_t)n * n), 256, 0, s>>>(H, ldh, U, ldu, n, n);
    LAMQ_CHECK_LAUNCH("lamq_env_factor copy");
    env_prep_kernel<<<1, 1024, 0, s>>>(U, ldu, n, damp, dead);
    LAMQ_CHECK_LAUNCH("lamq_env_factor prep");
    flip_kernel<<<grid_for((int64_t)n * n), 256, 0, s>>>(U, ldu, F, n, n);
    LAMQ_CHECK_LAUNCH("lamq_env_factor flip");
    int st = chol_inv(s, F, n, X, n, n, W, status);
    if (st) return st;
    flip_kernel<<<grid_for((int64_t)n * n), 256, 0, s>>>(X, n, U, ldu, n);
    LAMQ_CHECK_LAUNCH("lamq_env_factor flip back");
    return LAMQ_OK;
}

extern "C" size_t lamq_cross_apply_workspace_size(int rows, int n) {
    if (rows <= 0 || n <= 0) return 0;
    return 2 * (size_t)rows * n * sizeof(double);
}

extern "C" int lamq_cross_apply(const double *W, int64_t ldw, int rows, int n, const double *D, int64_t ldd,
                                const double *Linv, int64_t ldl, double alpha, double *out, int64_t ldo,
                                void *workspace, size_t workspace_bytes, lamq_stream_t stream) {
    LAMQ_REQUIRE(rows >= 0 && n >= 0 && ldd >= n && ldl >= n && ldo >= n && (W == nullptr || ldw >= n),
                 "lamq_cross_apply: bad shape");
    LAMQ_REQUIRE(W != nullptr || rows == n, "lamq_cross_apply: W = NULL (the identity) needs rows == n");
    if (rows == 0 || n == 0) return LAMQ_OK;
    LAMQ_REQUIRE(D && Linv && out && workspace, "lamq_cross_apply: null pointer");
    LAMQ_REQUIRE(out != W && out != D, "lamq_cross_apply: out aliases an input");
    LAMQ_REQUIRE(workspace_bytes >= lamq_cross_apply_workspace_size(rows, n), "lamq_cross_apply: workspace too small");
    cudaStream_t s = (cudaStream_t)stream;
    double *P = reinterpret_cast<double *>(workspace);  // W·D
    double *P2 = P + (size_t)rows * n;                  // (W·D)·Linvᵀ
    const double *Pin = D;
    int64_t ldp = ldd;
    int st;
    if (W != nullptr) {
        st = dgemm(s, 0, rows, n, n, 1.0, W, ldw, D, ldd, 0.0, P, n);
        if (st) return st;
        Pin = P;
        ldp = n;
        copy_block_kernel<<<grid_for((int64_t)rows * n), 256, 0, s>>>(W, ldw, out, ldo, rows, n);
        LAMQ_CHECK_LAUNCH("lamq_cross_apply copy");
    } else {
        identity_kernel<<<grid_for((int64_t)n * n), 256, 0, s>>>(out, ldo, n);
        LAMQ_CHECK_LAUNCH("lamq_cross_apply identity");
    }
    // P2 = P·Linvᵀ: the stored B (Linv) is lower, so NT skips k > column
    st = dgemm(s, 1, rows, n, n, 1.0, Pin, ldp, Linv, ldl, 0.0, P2, n, 0, 0, 1);
    if (st) return st;
    // out += alpha·P2·Linv: NN with a lower B skips k < column
    return dgemm(s, 0, rows, n, n, alpha, P2, n, Linv, ldl, 1.0, out, ldo, 0, 0, 1);
}

extern "C" int lamq_ridge(const double *H, int64_t ldh, double *A, int64_t lda, int n, double lam,
                          lamq_stream_t stream) {
    LAMQ_REQUIRE(n >= 0 && ldh >= n && lda >= n, "lamq_ridge: bad shape");
    if (n == 0) return LAMQ_OK;
    LAMQ_REQUIRE(H && A, "lamq_ridge: null pointer");
    cudaStream_t s = (cudaStream_t)stream;
    copy_block_kernel<<<grid_for((int64_t)n * n), 256, 0, s>>>(H, ldh, A, lda, n, n);
    LAMQ_CHECK_LAUNCH("lamq_ridge copy");
    ridge_diag_kernel<<<1, 1024, 0, s>>>(A, lda, n, lam);
    LAMQ_CHECK_LAUNCH("lamq_ridge");
    return LAMQ_OK;
}

extern "C" size_t lamq_proxy_loss_workspace_size(int64_t rows, int n) {
    if (rows <= 0 || n <= 0) return 0;
    const size_t rb = (size_t)std::min<int64_t>(rows, kProxyRowBlock);
    return (2 * rb * (size_t)n + (size_t)rows) * sizeof(double);
}

extern "C" int lamq_proxy_loss(const double *Wq, int64_t ldq, const double *W, int64_t ldw, int64_t rows, int n,
                               const double *H, int64_t ldh, double *row_loss, double *total, void *workspace,
                               size_t workspace_bytes, lamq_stream_t stream) {
    LAMQ_REQUIRE(rows >= 0 && n >= 0 && ldq >= n && ldh >= n && (W == nullptr || ldw >= n),
                 "lamq_proxy_loss: bad shape");
    LAMQ_REQUIRE(rows <= INT_MAX, "lamq_proxy_loss: %lld rows exceed the product's range", (long long)rows);
    LAMQ_REQUIRE(total != nullptr, "lamq_proxy_loss: null pointer");
    cudaStream_t s = (cudaStream_t)stream;
    if (rows == 0 || n == 0) return LAMQ_OK;  // the loss of an empty word is 0; nothing is written
    LAMQ_REQUIRE(Wq && H && workspace, "lamq_proxy_loss: null pointer");
    LAMQ_REQUIRE(workspace_bytes >= lamq_proxy_loss_workspace_size(rows, n), "lamq_proxy_loss: workspace too small");
    const int64_t rb = std::min<int64_t>(rows, kProxyRowBlock);
    double *E = reinterpret_cast<double *>(workspace);
    double *P = E + (size_t)rb * n;
    double *loss = row_loss ? row_loss : P + (size_t)rb * n;
    for (int64_t r0 = 0; r0 < rows; r0 += rb) {
        const int m = (int)std::min<int64_t>(rb, rows - r0);
        diff_kernel<<<grid_for((int64_t)m * n), 256, 0, s>>>(Wq + r0 * ldq, ldq, W ? W + r0 * ldw : nullptr, ldw, E,
                                                            m, n);
        LAMQ_CHECK_LAUNCH("lamq_proxy_loss difference");
        const int st = dgemm(s, 0, m, n, n, 1.0, E, n, H, ldh, 0.0, P, n);
        if (st) return st;
        row_dot_kernel<<<(m + 7) / 8, 256, 0, s>>>(P, E, m, n, loss + r0);
        LAMQ_CHECK_LAUNCH("lamq_proxy_loss rows");
    }
    sum_rows_kernel<<<1, 256, 0, s>>>(loss, rows, total);
    LAMQ_CHECK_LAUNCH("lamq_proxy_loss total");
    return LAMQ_OK;
}
