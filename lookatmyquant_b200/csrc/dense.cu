// Dense fp64 linear algebra on the fp64 tensor cores (mma.sync m8n8k4 f64): the GEMM, blocked Cholesky and
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
// GEMM: 128 × 64 CTA tiles, 8 warps of 32 × 32, K in steps of 16 staged through shared memory by cp.async (double
// buffered, rows padded so every fragment load is bank-conflict free); a triangular operand clips each tile's K range.
// Cholesky and inverse together, recursively: (L11, X11) = rec(A11), L21 = A21·X11ᵀ, A22 −= L21·L21ᵀ,
// (L22, X22) = rec(A22), X21 = −X22·(L21·X11) — 0.58n³ multiply-adds in large GEMMs; 128 x 128 leaves are factored
// and inverted in one CTA's shared memory.
#include <algorithm>
#include <vector>

#include "lamq_common.cuh"

namespace lamq {

namespace {

constexpr int GM = 128, GN = 128, GK = 16, GSTAGES = 4;
constexpr int kGemmWarpsM = 2, kGemmWarpsN = 4;  // 8 warps of 64 x 32
constexpr int kGemmThreads = 32 * kGemmWarpsM * kGemmWarpsN;
constexpr int WTM = GM / kGemmWarpsM, WTN = GN / kGemmWarpsN, FI = WTM / 16, FJ = WTN / 8;  // m16n8 tiles
constexpr int SA = GK + 4;   // A tile row stride (doubles): fragment loads hit every bank pair once
constexpr int SBN = GN + 4;  // B tile (k-major, NN) row stride
constexpr int SBT = GK + 4;  // B tile (n-major, NT) row stride
constexpr int NB = 128;      // Cholesky panel / diagonal block

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

__device__ __forceinline__ void dmma(double &c0, double &c1, double a, double b) {
    asm("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0, %1}, {%2}, {%3}, {%0, %1};"
                 : "+d"(c0), "+d"(c1)
                 : "d"(a), "d"(b));
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

// One thread's share of a tile copy, worked out once per CTA: slot q copies the element pair (r, c..c+1) of a
// rows x cols tile (cols even, 16-byte copies) or the single element (r, c) (8-byte copies) of a row-major source,
// zero-filling what lies outside Rmax x Cmax. Per K step only the K offset changes.
struct TileCopy {
    static constexpr int kSlots = 8;
    int n;                    // slots in use
    int soff[kSlots];         // destination offsets (doubles)
    int64_t goff[kSlots];     // source offsets (doubles) at K offset 0
    int rr[kSlots], cc[kSlots];
};

// `k_rows`: the tile's rows run along K (B without transposition), else its columns do.
__device__ __forceinline__ void tile_copy_init(TileCopy &t, int ld, int64_t lds, int r0, int c0, int rows, int cols,
                                               bool vec) {
    const int per = vec ? cols / 2 : cols;
    t.n = 0;
#pragma unroll
    for (int q = 0; q < TileCopy::kSlots; ++q) {
        const int e = threadIdx.x + q * kGemmThreads;
        const int r = e / per, c = vec ? 2 * (e % per) : e % per;
        t.soff[q] = r * ld + c;
        t.goff[q] = (int64_t)(r0 + r) * lds + c0 + c;
        t.rr[q] = r0 + r;
        t.cc[q] = c0 + c;
        if (e < rows * per) t.n = q + 1;
    }
}

// Issues the copies for a tile whose rows (k_rows) or columns are shifted by k0 along K.
__device__ __forceinline__ void tile_copy_issue(const TileCopy &t, double *dst, const double *src, int64_t lds, int k0,
                                                bool k_rows, int Rmax, int Cmax, bool vec) {
    const int64_t shift = k_rows ? (int64_t)k0 * lds : (int64_t)k0;
#pragma unroll
    for (int q = 0; q < TileCopy::kSlots; ++q) {
        if (q >= t.n) break;
        const int r = t.rr[q] + (k_rows ? k0 : 0), c = t.cc[q] + (k_rows ? 0 : k0);
        if (vec) {
            int nv = (r < Rmax) ? min(2, Cmax - c) : 0;
            nv = nv < 0 ? 0 : nv;
            cp16(dst + t.soff[q], src + (nv > 0 ? t.goff[q] + shift : 0), nv);
        } else {
            const bool ok = r < Rmax && c < Cmax;
            cp8(dst + t.soff[q], src + (ok ? t.goff[q] + shift : 0), ok);
        }
    }
}

constexpr int kATile = GM * SA;
constexpr int kBTile = GK * SBN > GN * SBT ? GK * SBN : GN * SBT;
constexpr size_t kGemmSmem = GSTAGES * (size_t)(kATile + kBTile) * sizeof(double);

// C = α·A·B(ᵀ) + β·C on the fp64 tensor cores: 128 x 128 CTA tiles, 8 warps of 64 x 32 (4 x 4 fragments of
// mma.sync m16n8k16 f64 — on B200 the large fp64 shape sustains ~37 TFLOP/s where m8n8k4 with changing operands
// stops near 32), K in steps of 16 through a 4-stage cp.async ring.
__global__ void __launch_bounds__(kGemmThreads) dgemm_kernel(GemmArgs g) {
    extern __shared__ __align__(16) double gsm[];
    const int m0 = blockIdx.y * GM, n0 = blockIdx.x * GN;
    if (g.lower_only && m0 + GM - 1 < n0) return;  // every row of the tile is above the diagonal
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int wm = (warp / kGemmWarpsN) * WTM, wn = (warp % kGemmWarpsN) * WTN;  // warp tile WTM x WTN
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
    TileCopy ca, cb;
    tile_copy_init(ca, SA, g.lda, m0, 0, GM, GK, vec);  // A: GM x GK at (m0, k)
    if (!g.transB) tile_copy_init(cb, SBN, g.ldb, 0, n0, GK, GN, vec);  // B: GK x GN at (k, n0)
    else tile_copy_init(cb, SBT, g.ldb, n0, 0, GN, GK, vec);            // B: GN x GK at (n0, k)
    auto load = [&](int s, int k0) {
        tile_copy_issue(ca, As(s), g.A, g.lda, k0, false, g.M, g.K, vec);
        if (!g.transB) tile_copy_issue(cb, Bs(s), g.B, g.ldb, k0, true, g.K, g.N, vec);
        else tile_copy_issue(cb, Bs(s), g.B, g.ldb, k0, false, g.N, g.K, vec);
    };
#pragma unroll
    for (int s = 0; s < GSTAGES - 1; ++s) {
        if (s < ksteps) load(s, kb + s * GK);
        asm volatile("cp.async.commit_group;" ::: "memory");
    }
    for (int ks = 0; ks < ksteps; ++ks) {
        asm volatile("cp.async.wait_group %0;" ::"n"(GSTAGES - 2) : "memory");
        __syncthreads();  // stage ks is in, and stage ks − 1 is free for the next load
        const int nxt = ks + GSTAGES - 1;
        if (nxt < ksteps) load(nxt % GSTAGES, kb + nxt * GK);
        asm volatile("cp.async.commit_group;" ::: "memory");
        const double *A = As(ks % GSTAGES), *B = Bs(ks % GSTAGES);
        double bf[FJ][4];
#pragma unroll
        for (int j = 0; j < FJ; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e)
                bf[j][e] = g.transB ? B[(wn + 8 * j + fg) * SBT + ft + 4 * e] : B[(ft + 4 * e) * SBN + wn + 8 * j + fg];
#pragma unroll
        for (int i = 0; i < FI; ++i) {
            double af[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) af[e] = A[(wm + 16 * i + fg + 8 * (e & 1)) * SA + ft + 4 * (e >> 1)];
#pragma unroll
            for (int j = 0; j < FJ; ++j) dmma16816(acc[i][j], af, bf[j]);
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

// Factors the nb x nb diagonal block at A[k0][k0] in place (lower Cholesky; the block's strict upper part set to zero)
// and writes its inverse to X[k0][k0] (lower, strict upper zero). A non-positive pivot sets *status = LAMQ_ERR_NOT_PD.
// 512 threads: thread t owns column t & 127 and every fourth row from t >> 7.
__global__ void __launch_bounds__(512) diag_block_kernel(double *A, int64_t lda, int k0, int nb, double *X,
                                                         int64_t ldx, int *status) {
    extern __shared__ __align__(16) double Bk[];  // nb x nb, row stride nb + 1
    const int ld = nb + 1;
    const int t = threadIdx.x, tc = t & 127, tg = t >> 7;
    for (int r = tg; r < nb; r += 4)
        if (tc < nb) Bk[r * ld + tc] = (tc <= r) ? A[(int64_t)(k0 + r) * lda + k0 + tc] : 0.0;
    __shared__ int bad;
    if (t == 0) bad = 0;
    __syncthreads();
    for (int j = 0; j < nb; ++j) {
        if (t == 0) {
            const double d = Bk[j * ld + j];
            if (!(d > 0.0)) bad = 1;
            Bk[j * ld + j] = sqrt(fmax(d, 0.0));
        }
        __syncthreads();
        const double dj = Bk[j * ld + j];
        // scale column j below the pivot
        for (int i = j + 1 + t; i < nb; i += 512) Bk[i * ld + j] = Bk[i * ld + j] / dj;
        __syncthreads();
        // trailing update of the lower part: B[i][c] -= B[i][j]·B[c][j] for j < c <= i
        if (tc > j && tc < nb) {
            const double bcj = Bk[tc * ld + j];
            for (int i = tc + ((tg - tc) & 3); i < nb; i += 4) Bk[i * ld + tc] -= Bk[i * ld + j] * bcj;
        }
        __syncthreads();
    }
    for (int r = tg; r < nb; r += 4)
        if (tc < nb) A[(int64_t)(k0 + r) * lda + k0 + tc] = (tc <= r) ? Bk[r * ld + tc] : 0.0;
    // inverse of the lower triangle by forward substitution, every column at once:
    //   X[i][c] = (δ_ic − Σ_{c<=k<i} L[i][k]·X[k][c]) / L[i][i]
    // four threads per column (k interleaved, a shuffle reduction per row). X[k][c] for k > c is kept transposed in the
    // strict upper triangle of the block (free after the factorization), X[c][c] in xd.
    __shared__ double xd[NB];
    {
        const int c = t >> 2, part = t & 3;
        const bool active = c < nb;
        if (active && part == 0) xd[c] = 1.0 / Bk[c * ld + c];
        __syncwarp();
        for (int i = 1; i < nb; ++i) {
            double a0 = 0.0, a1 = 0.0;
            if (active && i > c) {
                int k = c + part;
                for (; k + 4 < i; k += 8) {
                    a0 = fma(Bk[i * ld + k], (k == c) ? xd[c] : Bk[c * ld + k], a0);
                    a1 = fma(Bk[i * ld + k + 4], Bk[c * ld + k + 4], a1);
                }
                if (k < i) a0 = fma(Bk[i * ld + k], (k == c) ? xd[c] : Bk[c * ld + k], a0);
            }
            double acc = a0 + a1;
            acc += __shfl_xor_sync(0xffffffffu, acc, 1);
            acc += __shfl_xor_sync(0xffffffffu, acc, 2);
            if (active && part == 0 && i > c) Bk[c * ld + i] = -acc / Bk[i * ld + i];
            __syncwarp();
        }
    }
    __syncthreads();
    for (int r = tg; r < nb; r += 4)
        if (tc < nb) X[(int64_t)(k0 + r) * ldx + k0 + tc] = (tc < r) ? Bk[tc * ld + r] : (tc == r ? xd[r] : 0.0);
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

int grid_for(int64_t n) { return (int)std::min<int64_t>((n + 255) / 256, 148 * 16); }

int dgemm(cudaStream_t s, int transB, int M, int N, int K, double alpha, const double *A, int64_t lda,
          const double *B, int64_t ldb, double beta, double *C, int64_t ldc, int lower_only = 0, int a_lower = 0,
          int b_lower = 0) {
    if (M <= 0 || N <= 0) return LAMQ_OK;
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(dgemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGemmSmem);
        attr = true;
    }
    const bool vec = ((uintptr_t)A % 16 == 0) && (lda % 2 == 0) && ((uintptr_t)B % 16 == 0) && (ldb % 2 == 0);
    GemmArgs g{M, N, K, alpha, beta, A, lda, B, ldb, C, ldc, transB, lower_only, a_lower, b_lower, vec ? 1 : 0};
    dim3 grid((N + GN - 1) / GN, (M + GM - 1) / GM);
    dgemm_kernel<<<grid, kGemmThreads, kGemmSmem, s>>>(g);
    LAMQ_CHECK_LAUNCH("dgemm");
    return LAMQ_OK;
}

// Recursive Cholesky with inverse of the block [o, o+m) of A (lower part read): L overwrites A's lower part, L⁻¹ goes
// to X's lower part. [[A11, ·], [A21, A22]]: (L11, X11) = rec(A11); L21 = A21·X11ᵀ; A22 -= L21·L21ᵀ;
// (L22, X22) = rec(A22); X21 = −X22·(L21·X11). W has room for (m/2 + NB) x m/2 doubles.
int chol_inv_rec(cudaStream_t s, double *A, int64_t lda, double *X, int64_t ldx, int o, int m, double *W, int *status) {
    if (m <= NB) {
        diag_block_kernel<<<1, 512, m * (m + 1) * sizeof(double), s>>>(A, lda, o, m, X, ldx, status);
        LAMQ_CHECK_LAUNCH("diagonal block");
        return LAMQ_OK;
    }
    const int nblk = (m + NB - 1) / NB;
    const int m1 = (nblk / 2) * NB, m2 = m - m1;
    int st = chol_inv_rec(s, A, lda, X, ldx, o, m1, W, status);
    if (st) return st;
    double *A21 = A + (int64_t)(o + m1) * lda + o;
    double *A22 = A + (int64_t)(o + m1) * lda + o + m1;
    double *X11 = X + (int64_t)o * ldx + o;
    double *X21 = X + (int64_t)(o + m1) * ldx + o;
    double *X22 = X + (int64_t)(o + m1) * ldx + o + m1;
    // L21 = A21·X11ᵀ (X11 lower), staged in X21 then copied over A21
    st = dgemm(s, 1, m2, m1, m1, 1.0, A21, lda, X11, ldx, 0.0, X21, ldx, 0, 0, 1);
    if (st) return st;
    copy_block_kernel<<<grid_for((int64_t)m2 * m1), 256, 0, s>>>(X21, ldx, A21, lda, m2, m1);
    LAMQ_CHECK_LAUNCH("panel copy");
    // A22 -= L21·L21ᵀ (lower part)
    st = dgemm(s, 1, m2, m2, m1, -1.0, A21, lda, A21, lda, 1.0, A22, lda, 1);
    if (st) return st;
    st = chol_inv_rec(s, A, lda, X, ldx, o + m1, m2, W, status);
    if (st) return st;
    // X21 = −X22·(L21·X11): X11 and X22 lower triangular
    st = dgemm(s, 0, m2, m1, m1, 1.0, A21, lda, X11, ldx, 0.0, W, m1, 0, 0, 1);
    if (st) return st;
    return dgemm(s, 0, m2, m1, m2, -1.0, X22, ldx, W, m1, 0.0, X21, ldx, 0, 1, 0);
}

int chol_inv(cudaStream_t s, double *A, int64_t lda, double *X, int64_t ldx, int n, double *W, int *status) {
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(diag_block_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)(NB * (NB + 1) * sizeof(double)));
        attr = true;
    }
    int st = chol_inv_rec(s, A, lda, X, ldx, 0, n, W, status);
    if (st) return st;
    zero_upper_kernel<<<grid_for((int64_t)n * n), 256, 0, s>>>(A, lda, n);
    LAMQ_CHECK_LAUNCH("zero upper");
    zero_upper_kernel<<<grid_for((int64_t)n * n), 256, 0, s>>>(X, ldx, n);
    LAMQ_CHECK_LAUNCH("zero upper");
    return LAMQ_OK;
}

size_t w_elems(int n) { return (size_t)((n + 1) / 2 + NB) * (size_t)((n + 1) / 2 + NB); }

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
