/* CPU restatement of the segmented min-plus Viterbi of trellis.py:84-105
 * (identical to qat.py:141-152): TEST INFRASTRUCTURE ONLY.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU legs load this
 * library, as the checker; the product library never does.
 *
 * Per sequence x (T float32 values), with Q = 2^(L-R), K = 2^R:
 *   cost_0[s] = (x_0 - cw[s])^2
 *   for t >= 1:  m[q]  = min_k cost_{t-1}[k*Q + q]     (first k on ties,
 *                bp[t][q] = that k                        torch.min(dim=1))
 *                cost_t[s] = (x_t - cw[s])^2 + m[s >> R]
 *   s_{T-1} = first argmin of cost_{T-1}                 (torch.argmin)
 *   s_{t-1} = bp[t][s_t >> R] * Q + (s_t >> R)
 *
 * Every value is a float32 sub, then a float32 multiply, then a float32 add,
 * each rounded to nearest (torch's separate tensor ops on the CPU): the file
 * is compiled with -ffp-contract=off and without fast-math so the compiler
 * fuses nothing.  Ties keep the lower index because only a strictly smaller
 * cost replaces the running minimum.  NaN inputs are outside the reference's
 * specification and are not handled specially.
 */
#include <stdint.h>
#include <stdlib.h>
#include <math.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* cost[q*K + j] = (xt - cw[q*K + j])^2 + m[q] for j < K (K a compile-time
 * constant after inlining): a float32 sub, multiply and add, each rounded */
static inline __attribute__((always_inline)) void step_costs(float *cost, const float *cw, const float *m, float xt,
                                                             int Q, const int K) {
    for (int q = 0; q < Q; ++q) {
        const float mq = m[q];
        float *c = cost + (size_t)q * (size_t)K;
        const float *w = cw + (size_t)q * (size_t)K;
        for (int j = 0; j < K; ++j) {
            const float d = xt - w[j];
            const float sq = d * d;
            c[j] = sq + mq;
        }
    }
}

static void viterbi_one(const float *x, int T, int L, int R, const float *cw, int32_t *out,
                        float *cost, float *m, uint8_t *bp) {
    const int S = 1 << L, Q = 1 << (L - R), K = 1 << R;
    const float x0 = x[0];
    for (int s = 0; s < S; ++s) {
        const float d = x0 - cw[s];
        cost[s] = d * d;
    }
    for (int t = 1; t < T; ++t) {
        uint8_t *b = bp + (size_t)(t - 1) * (size_t)Q;
        for (int q = 0; q < Q; ++q) {
            m[q] = cost[q];
            b[q] = 0;
        }
        for (int k = 1; k < K; ++k) {
            const float *c = cost + (size_t)k * (size_t)Q;
            for (int q = 0; q < Q; ++q) {
                const int lt = c[q] < m[q];
                m[q] = lt ? c[q] : m[q];
                b[q] = lt ? (uint8_t)k : b[q];
            }
        }
        const float xt = x[t];
        switch (R) {
            case 1: step_costs(cost, cw, m, xt, Q, 2); break;
            case 2: step_costs(cost, cw, m, xt, Q, 4); break;
            case 3: step_costs(cost, cw, m, xt, Q, 8); break;
            case 4: step_costs(cost, cw, m, xt, Q, 16); break;
            default:
                for (int s = 0; s < S; ++s) {
                    const float d = xt - cw[s];
                    const float sq = d * d;
                    cost[s] = sq + m[s >> R];
                }
        }
    }
    int best = 0;
    float bv = cost[0];
    for (int s = 1; s < S; ++s)
        if (cost[s] < bv) { bv = cost[s]; best = s; }
    out[T - 1] = best;
    int s = best;
    for (int t = T - 1; t >= 1; --t) {
        const int q = s >> R;
        s = (int)bp[(size_t)(t - 1) * (size_t)Q + (size_t)q] * Q + q;
        out[t - 1] = s;
    }
}

/* Viterbi state paths of nseq sequences (rows of xn, T values each) into
 * states (nseq, T) int32.  threads <= 0: the OpenMP default.  Returns 0, or
 * -1 on bad arguments / out of memory. */
int uq_oracle_viterbi(const float *xn, int64_t nseq, int T, int L, int R, const float *cw, int32_t *states,
                      int threads) {
    if (nseq < 0 || T < 1 || L < 1 || L > 20 || R < 1 || R > 8 || R > L || !xn || !cw || !states) return -1;
    const int S = 1 << L, Q = 1 << (L - R);
    int failed = 0;
#ifdef _OPENMP
    if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel num_threads(threads) reduction(| : failed)
#endif
    {
        float *cost = (float *)malloc(sizeof(float) * (size_t)S);
        float *m = (float *)malloc(sizeof(float) * (size_t)Q);
        uint8_t *bp = (uint8_t *)malloc((size_t)(T > 1 ? T - 1 : 1) * (size_t)Q);
        if (!cost || !m || !bp) {
            failed = 1;
        } else {
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
            for (int64_t i = 0; i < nseq; ++i)
                viterbi_one(xn + i * (int64_t)T, T, L, R, cw, states + i * (int64_t)T, cost, m, bp);
        }
        free(cost);
        free(m);
        free(bp);
    }
    return failed ? -1 : 0;
}

/* fp32 cost of a given state path under the same recurrence along the path:
 * acc_0 = (x_0 - cw[s_0])^2, acc_t = (x_t - cw[s_t])^2 + acc_{t-1}.  For the
 * Viterbi path this equals the minimum final cost, so two different paths
 * with equal path costs are an exact cost tie. */
float uq_oracle_path_cost(const float *x, const int32_t *st, int T, const float *cw) {
    float acc = 0.0f;
    for (int t = 0; t < T; ++t) {
        const float d = x[t] - cw[st[t]];
        const float sq = d * d;
        acc = t == 0 ? sq : sq + acc;
    }
    return acc;
}

/* The same Viterbi with each cost formed by one fused multiply-add,
 * fmaf(d, d, m) -- NOT the reference's arithmetic.  Test infrastructure for
 * the checker only: sequences on which it and uq_oracle_viterbi disagree are
 * the ones that expose a device whose compiler contracted the square and the
 * add into one rounding. */
static void viterbi_one_fused(const float *x, int T, int L, int R, const float *cw, int32_t *out,
                              float *cost, float *m, uint8_t *bp) {
    const int S = 1 << L, Q = 1 << (L - R), K = 1 << R;
    for (int s = 0; s < S; ++s) {
        const float d = x[0] - cw[s];
        cost[s] = d * d;
    }
    for (int t = 1; t < T; ++t) {
        uint8_t *b = bp + (size_t)(t - 1) * (size_t)Q;
        for (int q = 0; q < Q; ++q) {
            m[q] = cost[q];
            b[q] = 0;
        }
        for (int k = 1; k < K; ++k) {
            const float *c = cost + (size_t)k * (size_t)Q;
            for (int q = 0; q < Q; ++q) {
                const int lt = c[q] < m[q];
                m[q] = lt ? c[q] : m[q];
                b[q] = lt ? (uint8_t)k : b[q];
            }
        }
        const float xt = x[t];
        for (int s = 0; s < S; ++s) {
            const float d = xt - cw[s];
            cost[s] = fmaf(d, d, m[s >> R]);
        }
    }
    int best = 0;
    float bv = cost[0];
    for (int s = 1; s < S; ++s)
        if (cost[s] < bv) { bv = cost[s]; best = s; }
    out[T - 1] = best;
    int s = best;
    for (int t = T - 1; t >= 1; --t) {
        const int q = s >> R;
        s = (int)bp[(size_t)(t - 1) * (size_t)Q + (size_t)q] * Q + q;
        out[t - 1] = s;
    }
}

int uq_oracle_viterbi_fused(const float *xn, int64_t nseq, int T, int L, int R, const float *cw, int32_t *states,
                            int threads) {
    if (nseq < 0 || T < 1 || L < 1 || L > 20 || R < 1 || R > 8 || R > L || !xn || !cw || !states) return -1;
    const int S = 1 << L, Q = 1 << (L - R);
    int failed = 0;
#ifdef _OPENMP
    if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel num_threads(threads) reduction(| : failed)
#endif
    {
        float *cost = (float *)malloc(sizeof(float) * (size_t)S);
        float *m = (float *)malloc(sizeof(float) * (size_t)Q);
        uint8_t *bp = (uint8_t *)malloc((size_t)(T > 1 ? T - 1 : 1) * (size_t)Q);
        if (!cost || !m || !bp) {
            failed = 1;
        } else {
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
            for (int64_t i = 0; i < nseq; ++i)
                viterbi_one_fused(xn + i * (int64_t)T, T, L, R, cw, states + i * (int64_t)T, cost, m, bp);
        }
        free(cost);
        free(m);
        free(bp);
    }
    return failed ? -1 : 0;
}
