/*
 * TEST INFRASTRUCTURE ONLY: CPU restatement of the reference's bitshift-trellis Viterbi, used as the parity
 * checker for the CUDA kernels. Nothing in the product links or loads this file.
 *
 * Restates opgraph/codes.py:151-181 (`viterbi`) exactly, in single precision as the reference computes it:
 *   - states s_t = (s_{t-1} * 2^k + b) mod 2^L, value values[s_t] (codes.py:152-153);
 *   - the cost of entry t is (x_t - C[s])^2 as one fp32 subtraction and one fp32 multiply (codes.py:164,172),
 *     added to the best predecessor cost with one fp32 add (codes.py:172). The file is compiled with
 *     -ffp-contract=off so no fused multiply-add changes the rounding;
 *   - predecessors of s are h * 2^(L-k) + (s >> k), h < 2^k; the minimum keeps the smallest h on ties, as
 *     torch.min(dim) does (codes.py:170);
 *   - with a start state, only the 2^k successors of that state are allowed at t = 0 (codes.py:165-167);
 *   - the final state is the first minimum over all states (torch.argmin, codes.py:173), then back-pointers are
 *     followed to t = 0 (codes.py:174-179).
 * Rows are independent, so they are split across OpenMP threads.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static void viterbi_row(const float *x, int T, const float *C, int L, int k, int has_start, int64_t start,
                        int64_t *out, float *cost, float *best, uint8_t *back) {
    const int S = 1 << L, nb = 1 << k, R = 1 << (L - k);
    for (int s = 0; s < S; ++s) {
        float d = x[0] - C[s];
        cost[s] = d * d;
    }
    if (has_start) {
        /* first = ((start << k) | b) & (S - 1): every other state starts at +inf */
        int64_t r0 = start & (R - 1);
        for (int s = 0; s < S; ++s)
            if ((s >> k) != r0) cost[s] = INFINITY;
    }
    for (int t = 1; t < T; ++t) {
        uint8_t *bt = back + (size_t)t * R;
        for (int r = 0; r < R; ++r) {
            float m = cost[r];
            int a = 0;
            for (int h = 1; h < nb; ++h) {
                float c = cost[h * R + r];
                if (c < m) { m = c; a = h; }
            }
            best[r] = m;
            bt[r] = (uint8_t)a;
        }
        float xt = x[t];
        for (int s = 0; s < S; ++s) {
            float d = xt - C[s];
            float sq = d * d;
            cost[s] = best[s >> k] + sq;
        }
    }
    int sbest = 0;
    float m = cost[0];
    for (int s = 1; s < S; ++s)
        if (cost[s] < m) { m = cost[s]; sbest = s; }
    int64_t s = sbest;
    out[T - 1] = s;
    for (int t = T - 1; t > 0; --t) {
        int64_t r = s >> k;
        s = r + (int64_t)back[(size_t)t * R + r] * R;
        out[t - 1] = s;
    }
}

/* X: rows x T fp32 (row-major); C: 2^L fp32; start: rows int64 or NULL; out: rows x T int64. Returns 0. */
int oracle_viterbi(const float *X, int64_t rows, int T, const float *C, int L, int k, const int64_t *start,
                   int64_t *out) {
    if (T <= 0 || rows <= 0) return 0;
    const int S = 1 << L, R = 1 << (L - k);
#pragma omp parallel
    {
        float *cost = (float *)malloc(sizeof(float) * S);
        float *best = (float *)malloc(sizeof(float) * R);
        uint8_t *back = (uint8_t *)malloc((size_t)T * R);
#pragma omp for schedule(dynamic, 4)
        for (int64_t i = 0; i < rows; ++i)
            viterbi_row(X + i * T, T, C, L, k, start != NULL, start ? start[i] : 0, out + i * T, cost, best, back);
        free(cost);
        free(best);
        free(back);
    }
    return 0;
}
