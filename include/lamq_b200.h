/*
 * lamq_b200 — C ABI of the B200 (sm_100a) kernels for LookAtMyQuant's quantization-build hot path.
 *
 * Every entry point takes plain device pointers and sizes, runs asynchronously on the given CUDA stream and returns an
 * int status (LAMQ_OK = 0). The caller owns every buffer; entry points that need scratch take a caller-provided
 * workspace whose size a *_workspace_size() query returns, and allocate nothing themselves. Row-major layouts
 * throughout; `ld*` arguments are leading dimensions in elements.
 *
 * Reference interfaces replaced (ShinMegamiBoson/lookatmyquant, file:line):
 *   lamq_viterbi           opgraph/codes.py:151-181   viterbi(X, values, L, k, chunk=None, start=None)
 *   lamq_ldlq_rowtrellis   opgraph/syntax.py:86-124   sweep(W, env, project, width=16, lazy=128) with the project of
 *                          opgraph/codes.py:442-450 and RowTrellisCode.step (codes.py:397-404)
 *   lamq_ldlq_coltrellis   opgraph/syntax.py:86-124   the same sweep with TrellisCode.project (codes.py:363-383)
 *   lamq_xtx_accumulate,   quantize.py:1412-1470      H += Xᵀ(w⊙X), D += X_refᵀ(w⊙X) per calibration chunk, then
 *   lamq_weighted_split,                              H/n_tok and D/n_tok − H in fp64 (inline in quantize_stage);
 *   lamq_hessian_finalize  compiler.py:233-265        the unweighted H of `capture`
 *   lamq_rht_rows,         opgraph/codes.py:97-132    rht(n, seed) applied as X = W·R_inᵀ (:430), Hr = R_in·H·R_inᵀ
 *   lamq_transpose_f64                                (:439) and W_q = (S⊙V)·R_in, without forming R
 *   lamq_env_factor        opgraph/frame.py:515-522   Environment(H, damp): dead inputs, damping, U
 *   lamq_proxy_loss        quantize.py:1320-1325      best_word's error (E @ H * E).sum(), E = word − target
 *   lamq_cholesky_inverse_lower, lamq_ridge, lamq_dgemm, lamq_cross_apply
 *                          quantize.py:1330-1335      cross_target: M = I + α·(solve(H + λ·mean(diag H)·I, Dᵀ))ᵀ
 *                          quantize.py:1503           target = W @ M
 *   lamq_pack_trellis,     compiler_artifact.py:225-297  pack_trellis / unpack_trellis (valid_path checked on pack)
 *   lamq_unpack_trellis
 *   lamq_decode_trellis    compiler_artifact.py:433-442  decode_rotated: table[state]·scale per group row
 *   lamq_trellis_product   runtime_mlx/fast_q35.py:69-172 the product kernel: y = S ⊙ (V[state]·(R_in x)) per group
 *   lamq_trellis_product_groups                       the same for all row groups that read one input, one launch
 *   lamq_trellis_gemm      fast_q35.py:69-201 with    many input vectors: the decode fused into a tcgen05 GEMM
 *                          compiler_artifact.py:433-442
 *   lamq_square_sums       row_importance.py:57-93,   per-channel E[y²], E[g²] (row importance) and per-token Σ g²
 *                          quantize.py:853-894        (GuidedQuant token weights)
 *   lamq_kl_reference,     compiler.py:176-187        the KL probe: ref_lp once, then per probe the KL of the held
 *   lamq_kl_head                                      positions' log_softmax(lm_head(h)) to it
 */
#ifndef LAMQ_B200_H
#define LAMQ_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *lamq_stream_t; /* a cudaStream_t; NULL is the legacy default stream */

enum {
    LAMQ_OK = 0,
    LAMQ_ERR_INVALID = 1,   /* bad shape, width, pointer or workspace size */
    LAMQ_ERR_CUDA = 2,      /* a CUDA launch or runtime error (lamq_last_error() has the text) */
    LAMQ_ERR_NOT_PD = 3,    /* a matrix was not positive definite even with the reference's extra damping */
    LAMQ_ERR_TIMEOUT = 4,   /* a bounded device-side wait gave up */
    LAMQ_ERR_NOT_PATH = 5   /* states are not a path through the trellis */
};

/* Version of this ABI (incremented on any signature change). */
int lamq_abi_version(void);

/* Text of the last error raised on the calling host thread ("" if none). */
const char *lamq_last_error(void);

/* Kernels this library has launched in the process (all threads): what a benchmark counts as its own launches. */
uint64_t lamq_kernel_launches(void);

/*
 * Viterbi over a bitshift trellis (opgraph/codes.py:151-181).
 * X: rows x T fp32 (ldX = T); values: 2^L fp32 table; start: rows int64 states or NULL (free start);
 * states: rows x T int64 out. Supported: L = 12, k in 1..4, T >= 1.
 * Each row's costs are fp32 and rounded exactly as the reference's tensor ops; ties go to the smallest predecessor and
 * the smallest final state, so the states are identical to the reference's.
 * workspace: lamq_viterbi_workspace_size(rows, T, L, k) bytes of device memory (the back-pointers); 0 when the call
 * needs none (T <= 32, or longer sequences whose warp-pair decoder keeps its back-pointers in shared memory on the
 * current device). Shapes whose back-pointers would overflow a size_t are rejected with LAMQ_ERR_INVALID.
 */
size_t lamq_viterbi_workspace_size(int64_t rows, int T, int L, int k);
int lamq_viterbi(const float *X, int64_t rows, int T, const float *values, int L, int k, const int64_t *start,
                 int64_t *states, void *workspace, size_t workspace_bytes, lamq_stream_t stream);

/*
 * lamq_viterbi without a workspace: no counterpart in the reference (its Viterbi is a PyTorch loop). For callers that
 * cannot allocate device memory — a host application whose own pool owns the whole device and forbids library
 * allocations, or an FFI binding (cgo, JNI, N-API) with no device allocator to take a workspace from. Same inputs,
 * outputs and states as lamq_viterbi; it calls no cudaMalloc, cudaFree or allocating library routine. Sequences
 * longer than 32 entries keep their back-pointers in a LAMQ_VITERBI_NOALLOC_SCRATCH_BYTES (32 MiB) array built into
 * the library's device image, so rows x T may be at most 131072 when T > 32 (larger inputs are rejected with
 * LAMQ_ERR_INVALID); sequences of at most 32 entries need no scratch and have no limit. The call runs on the current
 * device; its first call on each device looks up the array's device address, so make that first call before any
 * stream capture. All calls on a device share the array: calls whose kernels overlap on the GPU race on it.
 */
#define LAMQ_VITERBI_NOALLOC_SCRATCH_BYTES ((size_t)32 << 20)
int lamq_viterbi_noalloc(const float *X, int64_t rows, int T, const float *values, int L, int k,
                         const int64_t *start, int64_t *states, lamq_stream_t stream);

/*
 * Scalar-level LDLQ rounding in fp64 (opgraph/ldlq_gpu.py:29-49, `ldlq_round`; used by nested.py:117-119): X (rows x n,
 * in place, the inputs after each block receive the block's errors) is rounded input by input to the nearest of the
 * sorted `levels` (the bucketize of ldlq_gpu.py:35-41: ties to the lower level), each error e = (x − q) / U[j][j]
 * carried into the block's later inputs through U's row, and after each block of `block` (<= 128) inputs into the rest
 * through one product. Q (rows x n) receives the chosen levels. Workspace: lamq_ldlq_round_workspace_size(rows).
 */
size_t lamq_ldlq_round_workspace_size(int64_t rows);
int lamq_ldlq_round(double *X, int64_t ldX, int64_t rows, int n, const double *U, int64_t ldU, const double *levels,
                    int nlevels, int block, double *Q, int64_t ldQ, void *workspace, size_t workspace_bytes,
                    lamq_stream_t stream);

/*
 * The block-LDLQ sweep with a row trellis as its projection (opgraph/syntax.py:86-124 with codes.py:397-404,442-450):
 * the lm2 build's per-matrix hot loop, fused into one persistent kernel: tiles of 16 rows of one width per CTA, the
 * trellis decode per warp, the end-of-run refit on fp64 tensor cores.
 *
 * T:        rows x n fp64 (ldT), in/out. On entry the targets in the rotated basis (X = W·R_inᵀ); columns flagged in
 *           `dead` are zeroed first (syntax.py:100-101). On exit each column as it stood just before it was settled —
 *           what `sweep` returns.
 * U:        n x n fp64 (ldU), the upper Cholesky factor of H⁻¹ (frame.py:522).
 * dead:     n bytes (nonzero = dead input) or NULL.
 * S:        rows fp64, each row's RMS scale (codes.py:436).
 * tables:   4 x 2^L fp64: the trellis values for k = 1, 2, 3, 4 (row of k at (k-1)·2^L).
 * row_bits: rows bytes, each row's k in 1..4 (the row plan's widths); NULL means every row uses `k_all`.
 * width, look, lazy: RowTrellisCode's width and look-ahead and sweep's lazy run (16, 8, 128 in the reference);
 *           width + look <= 24, lazy a multiple of width.
 * states:   rows x n int16 out (ldStates = n): the trellis states.
 * settled:  rows x n fp64 out or NULL: the settled table values, in units of the row scale.
 * workspace: lamq_ldlq_rowtrellis_workspace_size(rows, n) bytes of device memory (the rows grouped by width into
 *           tiles, per-run tile counters, each row's last state, and the run's z per row: about rows x 1 KiB).
 * Supported: L = 12; width + look <= 24; lazy <= 128 and a multiple of 4.
 */
size_t lamq_ldlq_rowtrellis_workspace_size(int64_t rows, int n);
int lamq_ldlq_rowtrellis(double *T, int64_t ldT, int64_t rows, int n, const double *U, int64_t ldU,
                         const uint8_t *dead, const double *S, const double *tables, const uint8_t *row_bits, int k_all,
                         int L, int width, int look, int lazy, int16_t *states, double *settled, void *workspace,
                         size_t workspace_bytes, lamq_stream_t stream);

/*
 * The column-trellis LDLQ sweep: sweep (opgraph/syntax.py:86-124) with TrellisCode.project (opgraph/codes.py:363-383),
 * the `measure` path's trellis words. Per block of `width` columns, each column is cut into runs of Tm consecutive rows
 * and every run goes onto its nearest free-start trellis path (fp32 costs of T/S, as lamq_viterbi); then the block
 * LDLQ refit under U as in lamq_ldlq_rowtrellis.
 * T:        rows x n fp64, in: the target X (rotated on both sides); out: each column as it stood just before it was
 *           settled (sweep's return value).
 * table:    2^L fp64 trellis values of this k.
 * states:   rows x n int16 out; settled: rows x n fp64 out or NULL (table values, units of the row scale).
 * workspace: lamq_ldlq_coltrellis_workspace_size(rows, n, Tm, L, k, width, lazy) bytes.
 * Supported: L = 12, k in 1..4, rows a multiple of Tm, width <= 32, lazy a multiple of width.
 */
size_t lamq_ldlq_coltrellis_workspace_size(int64_t rows, int n, int Tm, int L, int k, int width, int lazy);
int lamq_ldlq_coltrellis(double *T, int64_t ldT, int64_t rows, int n, const double *U, int64_t ldU, const uint8_t *dead,
                         const double *S, const double *table, int k, int L, int Tm, int width, int lazy,
                         int16_t *states, double *settled, void *workspace, size_t workspace_bytes,
                         lamq_stream_t stream);

/*
 * Tensor-core contraction over tokens: acc[j][i] += Σ_t A[t][i]·B[t][j] (bf16 in, fp32 accumulate) for i, j < d.
 * A, B: tokens x d bf16 (raw 16-bit words), row-major with leading dimensions lda, ldb (multiples of 8, 16-byte
 * aligned). acc: d x d fp32 (ldacc), accumulated into (zero it before the first call). The sum is accumulated on chip
 * over chunks of `chunk_tokens` tokens (a multiple of 64) and each chunk's partial is added into acc, in chunk order
 * for every element: the result is bit-reproducible for a given call sequence. Where a tile's chunks run on several
 * CTAs at once (the last wave of tiles), their partials go through scratch taken stream-ordered from a memory pool the
 * library keeps per device (at most chunks x 74 tiles x 256 KiB) and are added after the launch.
 * symmetric != 0 (A and B the same tokens, C symmetric): only the blocks of rows j >= columns i are computed; read
 * the result through lamq_hessian_finalize. status: a device int, 0 on entry; a bounded device wait that gives up
 * sets it to LAMQ_ERR_TIMEOUT (then the result is invalid). H = XᵀX is A = B = X; the QEP moment D = X_refᵀX is A = X,
 * B = X_ref (acc then holds D itself).
 */
int lamq_xtx_accumulate(const uint16_t *A, int64_t lda, const uint16_t *B, int64_t ldb, int64_t tokens, int d,
                        int symmetric, float *acc, int64_t ldacc, int64_t chunk_tokens, int *status,
                        lamq_stream_t stream);

/*
 * lamq_xtx_accumulate with the products scaled: acc[j][i] += scale·Σ_t A[t][i]·B[t][j] (each chunk's fp32 partial is
 * multiplied by `scale` as it is added). With the tokens of one weight value w gathered, scale = w − 1 adds their
 * weighted share exactly from bf16 products (quantize.py:1389-1391).
 */
int lamq_xtx_accumulate_scaled(const uint16_t *A, int64_t lda, const uint16_t *B, int64_t ldb, int64_t tokens, int d,
                               int symmetric, float scale, float *acc, int64_t ldacc, int64_t chunk_tokens, int *status,
                               lamq_stream_t stream);

/* dst row r = src row idx[r] for r < n: bf16 rows of d (a multiple of 8) values, 16-byte aligned. */
int lamq_gather_rows(const uint16_t *src, int64_t lds, const int32_t *idx, int64_t n, int d, uint16_t *dst,
                     lamq_stream_t stream);

/*
 * Token weights (quantize.py:1389-1391, 593-629): the weighted tokens' share Σ_t (w_t − 1)·x_t ⊗ y_t as two extra
 * rows per token for lamq_xtx_accumulate. For each r < nw, t = idx[r]: out_split row r = hi, row r + nw = lo of
 * (w[t] − 1)·scaled[t] (fp32; hi = bf16(y), lo = bf16(y − hi)); out_plain rows r and r + nw = plain[t].
 * out_split and out_plain: 2·nw x d bf16 (leading dimension d).
 */
int lamq_weighted_split(const uint16_t *scaled, int64_t lds, const uint16_t *plain, int64_t ldp, const float *w,
                        const int32_t *idx, int64_t nw, int d, uint16_t *out_split, uint16_t *out_plain,
                        lamq_stream_t stream);

/* H[r][c] = accH[max(r,c)][min(r,c)] / n_tok (fp64, symmetric); with accD, D = accD / n_tok − H. d x d outputs. */
int lamq_hessian_finalize(const float *accH, const float *accD, int d, int64_t ld, double n_tok, double *H, double *D,
                          lamq_stream_t stream);

/*
 * Randomized Hadamard transform of each row (opgraph/codes.py:97-132, applied at codes.py:430,439): for every row v
 * of `in` (rows x n, n = a·b), out = scale · post ⊙ ((Ae ⊗ Be)·(pre ⊙ v)), with Ae (a x a) and Be (b x b) ±1
 * matrices given as row-wise sign bits (abits: a x ceil(a/32) words, bit k of word w of row p set when
 * Ae[p][32w + k] = -1; bbits likewise) and pre/post sign vectors of length n (or NULL). R = (A⊗B)/√n·diag(s) is
 * Ae = A, Be = B, pre = s, scale = 1/√n; Rᵀ is Ae = Aᵀ, Be = Bᵀ, post = s. in may equal out. Orders a, b <= 256.
 */
int lamq_rht_rows(const double *in, int64_t ldi, double *out, int64_t ldo, int64_t rows, int a, int b,
                  const uint32_t *abits, const uint32_t *bbits, const double *pre, const double *post, double scale,
                  lamq_stream_t stream);

/* out (cols x rows) = transpose of in (rows x cols), fp64; in and out must not alias. */
int lamq_transpose_f64(const double *in, int64_t ldi, double *out, int64_t ldo, int rows, int cols,
                       lamq_stream_t stream);

/*
 * fp64 on the tensor cores. C = α·A·B + β·C (transB = 0, B is K x N) or C = α·A·Bᵀ + β·C (transB = 1, B is N x K),
 * row-major.
 */
int lamq_dgemm(int transB, int M, int N, int K, double alpha, const double *A, int64_t lda, const double *B,
               int64_t ldb, double beta, double *C, int64_t ldc, lamq_stream_t stream);

/*
 * The proxy loss of quantize.py:1320-1325 (best_word: E = net.matrix() − target, err = (E @ H * E).sum()):
 * row_loss[r] = Σ_ij E[r][i]·H[i][j]·E[r][j] for E = Wq − W (W NULL: E = Wq), and *total = Σ_r row_loss[r] summed in a
 * fixed order (deterministic). All fp64, rows x n row-major; E·H runs on the fp64 tensor cores in blocks of 4096
 * rows. row_loss may be NULL. Workspace: lamq_proxy_loss_workspace_size(rows, n). With rows or n zero the loss is 0
 * and the call returns LAMQ_OK without touching the device (nothing is written to *total).
 */
size_t lamq_proxy_loss_workspace_size(int64_t rows, int n);
int lamq_proxy_loss(const double *Wq, int64_t ldq, const double *W, int64_t ldw, int64_t rows, int n, const double *H,
                    int64_t ldh, double *row_loss, double *total, void *workspace, size_t workspace_bytes,
                    lamq_stream_t stream);

/* Workspace bytes for lamq_env_factor and lamq_cholesky_inverse_lower of order n. */
size_t lamq_factor_workspace_size(int n);

/*
 * A (n x n, symmetric positive definite, lower part read) is replaced by L⁻¹, L the lower Cholesky factor (strict
 * upper part zero). status (device int, 0 on entry) becomes LAMQ_ERR_NOT_PD on a non-positive pivot.
 */
int lamq_cholesky_inverse_lower(double *A, int64_t lda, int n, void *workspace, size_t workspace_bytes, int *status,
                                lamq_stream_t stream);

/*
 * Environment (opgraph/frame.py:515-522): dead inputs (zero diagonal) get a unit diagonal and are flagged in `dead`
 * (n bytes, or NULL), H += damp·mean(diag H)·I, and U (n x n, upper) = the upper Cholesky factor of H⁻¹, computed as
 * J·chol(J·H·J)⁻¹·J. H is not modified. status as for lamq_cholesky_inverse_lower.
 */
int lamq_env_factor(const double *H, int64_t ldh, int n, double damp, double *U, int64_t ldu, uint8_t *dead,
                    void *workspace, size_t workspace_bytes, int *status, lamq_stream_t stream);

/* Workspace bytes for lamq_cross_apply over `rows` rows of order n. */
size_t lamq_cross_apply_workspace_size(int rows, int n);

/*
 * The QEP target W·M of quantize.py:1330-1335 and :1503 without forming M:
 *   out = W + alpha·((W·D)·Linvᵀ)·Linv,   M = I + alpha·D·(Linvᵀ·Linv) = I + alpha·(solve(A, Dᵀ))ᵀ,
 * with Linv the inverse of the lower Cholesky factor of A = H + λ·mean(diag H)·I, lower triangular with a zero strict
 * upper part as lamq_cholesky_inverse_lower leaves it (the two triangular products skip its zero blocks and cost
 * half a GEMM each). W is rows x n; with W = NULL it is the identity (rows must equal n) and out = M. out may not
 * alias W or D.
 */
int lamq_cross_apply(const double *W, int64_t ldw, int rows, int n, const double *D, int64_t ldd, const double *Linv,
                     int64_t ldl, double alpha, double *out, int64_t ldo, void *workspace, size_t workspace_bytes,
                     lamq_stream_t stream);

/* A = H + lam·mean(diag H)·I (quantize.py:1334). */
int lamq_ridge(const double *H, int64_t ldh, double *A, int64_t lda, int n, double lam, lamq_stream_t stream);

/*
 * The KL probe's head (compiler.py:176-187): logits z = H·Eᵀ of held positions (H: ntok x d final hidden states, E: V x
 * d LM head, bf16, K contiguous; the logits rounded to bf16 as the model's lm_head returns them), their log-softmax
 * and the KL to a reference distribution, in tcgen05 passes over the vocabulary that write no logits.
 * lamq_kl_reference (once per held set): from the reference model's H, writes the reference distribution
 *   pdist = softmax(z_ref) (ntok x V fp32, leading dimension ldp, rows 16-byte aligned), lse_ref (ntok fp32) and the
 *   per-position sums stat_a = Σ_v p·z_ref, stat_p = Σ_v p (fp64).
 * lamq_kl_head (every probe): KL_t = Σ_v p·(log p − log_softmax(z)) = A − B + (lse − lse_ref)·P per position into
 *   kl_pos (fp32), and kl_out[0] = Σ w·KL / Σ w, kl_out[1] = Σ w·KL, kl_out[2] = Σ w (fp64; w NULL: all ones).
 * workspace: lamq_kl_workspace_size(ntok) bytes. status: device int, LAMQ_ERR_TIMEOUT if a bounded wait gave up.
 */
size_t lamq_kl_workspace_size(int64_t ntok);
int lamq_kl_reference(const uint16_t *H, int64_t ldh, int64_t ntok, int d, const uint16_t *E, int64_t lde, int V,
                      float *pdist, int64_t ldp, float *lse_ref, double *stat_a, double *stat_p, void *workspace,
                      size_t workspace_bytes, int *status, lamq_stream_t stream);
int lamq_kl_head(const uint16_t *H, int64_t ldh, int64_t ntok, int d, const uint16_t *E, int64_t lde, int V,
                 const float *pdist, int64_t ldp, const float *lse_ref, const double *stat_a, const double *stat_p,
                 const float *w, float *kl_pos, double *kl_out, void *workspace, size_t workspace_bytes, int *status,
                 lamq_stream_t stream);

/*
 * Packed trellis rows (opgraph-packed-1, compiler_artifact.py:225-297). A row of n states (L-bit states, k-bit
 * symbols, 1 <= k <= 8, k < L <= 12) is stored as the symbols state & (2^k − 1), padded forward with zeros to a
 * multiple of 32 columns, reversed, and packed little-endian k bits each: lamq_trellis_words_per_row(n, k) = ⌈n/32⌉·k
 * uint32 words per row, rows back to back.
 */
int64_t lamq_trellis_words_per_row(int n, int k);

/*
 * pack_trellis (compiler_artifact.py:276-284) of rows x n int16 states. status (device int, 0 on entry) becomes
 * LAMQ_ERR_NOT_PATH when a row is not a trellis path from state 0 (valid_path, :261-267); the words are written anyway.
 */
int lamq_pack_trellis(const int16_t *states, int64_t lds, int64_t rows, int n, int k, int L, uint32_t *codes,
                      int *status, lamq_stream_t stream);

/* unpack_trellis (compiler_artifact.py:287-297): the int16 states of packed rows. */
int lamq_unpack_trellis(const uint32_t *codes, int64_t rows, int n, int k, int L, int16_t *states, int64_t lds,
                        lamq_stream_t stream);

/*
 * decode_rotated (compiler_artifact.py:433-442) for one row group: out[map[r]][j] = table[state_rj]·scales[r] in fp32
 * (map NULL: row r). table has 2^L fp32 entries, scales one fp32 per group row.
 */
int lamq_decode_trellis(const uint32_t *codes, int64_t rows, int n, int k, int L, const float *scales,
                        const float *table, const uint32_t *map, float *out, int64_t ldo, lamq_stream_t stream);

/*
 * The product of one packed row group with nvec input vectors (runtime_mlx/fast_q35.py:69-172):
 * y[v][map[r]] = scales[r]·Σ_j table[state_rj]·x[v][j], fp32. x (nvec x n, leading dimension ldx) is the input
 * after the group's input rotation R_in; y rows have leading dimension ldy.
 */
int lamq_trellis_product(const uint32_t *codes, int64_t rows, int n, int k, int L, const float *scales,
                         const float *table, const uint32_t *map, const float *x, int64_t ldx, int nvec, float *y,
                         int64_t ldy, lamq_stream_t stream);

/*
 * One packed row group of a grouped product: `rows` packed rows of k-bit symbols (1 <= k <= 4) and L-bit states,
 * their scales and 2^L-entry fp32 table, the output row of each (map, or NULL for row r) and the output y (nvec rows
 * of leading dimension ldy). 64 bytes, no padding.
 */
typedef struct lamq_product_group {
    const uint32_t *codes;
    int64_t rows;
    int k, L;
    const float *scales;
    const float *table;
    const uint32_t *map;
    float *y;
    int64_t ldy;
} lamq_product_group;

/*
 * lamq_trellis_product for ngroups row groups that all read the same rotated input x (nvec x n): the row groups of
 * one matrix, or of every matrix of a stage (runtime_mlx/fast_q35.py's q/k/v and gate/up share their input), in one
 * launch per 32 groups and 8 vectors. Each output row equals lamq_trellis_product's bit for bit. `groups` is host
 * memory, read before the call returns.
 */
int lamq_trellis_product_groups(const lamq_product_group *groups, int ngroups, int n, const float *x, int64_t ldx,
                                int nvec, lamq_stream_t stream);

/*
 * One row group of a trellis-dequant GEMM: `rows` weight rows whose states come either from packed codes
 * (opgraph-packed-1, k-bit symbols, 1 <= k <= 4, L-bit states, codes = rows x lamq_trellis_words_per_row(n, k) words)
 * or from an int16 state matrix (states, rows x lds; codes NULL), the rows' fp32 scales, the 2^L-entry fp32 table, the
 * output row of each (map, or NULL for row r), the output y (nvec rows of leading dimension ldy, fp32 or bf16) and
 * the input the group multiplies: x (nvec x n bf16, leading dimension ldx, the input after the group's input
 * rotation). 104 bytes, no padding (`reserved` is ignored).
 */
typedef struct lamq_gemm_group {
    const uint32_t *codes;
    const int16_t *states;
    int64_t lds;
    int64_t rows;
    int k, L;
    const float *scales;
    const float *table;
    const uint32_t *map;
    void *y;
    int64_t ldy;
    const uint16_t *x;
    int64_t ldx;
    int n;
    int reserved;
} lamq_gemm_group;

/*
 * The trellis-dequant GEMM for many input vectors (runtime_mlx/fast_q35.py:69-201's product y = S ⊙ (V[state]·x), and
 * compiler_artifact.py:433-442's decode W = S·V[state]): y[v][map[r]] = scales[r]·Σ_j bf16(table[state_rj])·x[v][j]
 * with fp32 accumulation on the tensor cores (pairs of CTAs, 256 rows a tile). Up to 512 vectors the weights are
 * decoded from the states straight into shared memory, tile by tile, and never written out; from 513 vectors on they
 * are decoded once into the workspace as bf16 rows and loaded by TMA (the same products, bit for bit). Each group's x
 * is 16-byte aligned with ldx a multiple of 8; all groups take nvec vectors. Groups may read different inputs (a
 * layer's stages): one launch takes up to 16 groups over up to 4 inputs, the groups of the longest rows first.
 * y_bf16: 0 writes fp32 outputs, 1 bf16. workspace: lamq_trellis_gemm_workspace_size(groups, ngroups, nvec) bytes of
 * device memory, 16-byte aligned (0, and NULL allowed, up to 512 vectors). status (device int, 0 on entry) becomes
 * LAMQ_ERR_TIMEOUT if a device wait gives up. `groups` is host memory, read before the call returns.
 */
size_t lamq_trellis_gemm_workspace_size(const lamq_gemm_group *groups, int ngroups, int64_t nvec);
int lamq_trellis_gemm(const lamq_gemm_group *groups, int ngroups, int64_t nvec, int y_bf16, void *workspace,
                      size_t workspace_bytes, int *status, lamq_stream_t stream);

/* Element types of lamq_square_sums and lamq_rht_rows_act. */
#define LAMQ_F32 0
#define LAMQ_BF16 1
#define LAMQ_F64 2

/*
 * lamq_rht_rows for activations: the same y = scale · post ⊙ ((Ae ⊗ Be)·(pre ⊙ v)) per row, summed in fp32, reading
 * bf16, fp32 or fp64 rows (in_dtype) and writing bf16 or fp32 (out_dtype) — the input rotation of a product whose
 * operand is bf16 (the trellis GEMM, a probed piece), R_in x (codes.py:430's rotation applied to activations).
 * n = a·b up to 25,600; in and out must not alias.
 */
int lamq_rht_rows_act(const void *in, int in_dtype, int64_t ldi, void *out, int out_dtype, int64_t ldo, int64_t rows,
                      int a, int b, const uint32_t *abits, const uint32_t *bbits, const double *pre,
                      const double *post, double scale, lamq_stream_t stream);

/*
 * Sums of squares of x (rows x cols, leading dimension ld, fp32 or bf16) in fp64: col_acc[j] += Σ_r x[r][j]² (the
 * per-output-channel E[y²] and E[g²] of row importance, row_importance.py:57-93, summed over windows by accumulating)
 * and row_out[r] = Σ_j x[r][j]² (the per-token Σ of squared output gradients of GuidedQuant's token weights,
 * quantize.py:853-894). Either output may be NULL. Deterministic (fixed summation order). Workspace (column sums
 * only): lamq_square_sums_workspace_size(rows, cols) bytes.
 */
size_t lamq_square_sums_workspace_size(int64_t rows, int cols);
int lamq_square_sums(const void *x, int dtype, int64_t rows, int cols, int64_t ld, double *col_acc, double *row_out,
                     void *workspace, size_t workspace_bytes, lamq_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* LAMQ_B200_H */
