/* viterbi_oracle.c -- CPU restatement of the reference's trellis Viterbi.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * encoder; nothing in the product path links or calls it.  It is a plain,
 * unoptimised restatement of the reference algorithm
 * (SergiioB/exl3xpu-mixedk quantize/quantize.py):
 *
 *   viterbi                 quantize.py:218-320  (emit_mode "sq", V = 1)
 *   quantize_seq_tailbite   quantize.py:323-354
 *
 * and keeps its fp32 arithmetic order exactly:
 *   cost_0[s]   = fl(fl(lut[s] - x_0)^2)            (+ 0 / +inf boundary mask)
 *   best_i[j]   = min_w cost_{i-1}[j + w*S_PRE]     first index on ties
 *   cost_i[s]   = fl(fl(fl(lut[s] - x_i)^2) + best_i[s >> K])
 * Build with -ffp-contract=off (no FMA contraction) and without fast-math.
 *
 * Layout: X is [nseq][T] (one sequence per row), states are [nseq][T] int32.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef struct {
    float *cost;     /* [S] */
    float *best;     /* [S_PRE] */
    uint16_t *bp;    /* [T][S_PRE] */
} vit_ws;

static int ws_alloc(vit_ws *w, int L, int K, int T) {
    size_t S = (size_t)1 << L, SP = (size_t)1 << (L - K);
    w->cost = (float *)malloc(S * sizeof(float));
    w->best = (float *)malloc(SP * sizeof(float));
    w->bp = (uint16_t *)malloc((size_t)(T > 0 ? T : 1) * SP * sizeof(uint16_t));
    return (w->cost && w->best && w->bp) ? 0 : -1;
}

static void ws_free(vit_ws *w) {
    free(w->cost);
    free(w->best);
    free(w->bp);
}

static inline float emit_sq(float f, float x) {
    float d = f - x;   /* fl(f - x) */
    return d * d;      /* fl(d * d); contraction is disabled at build time */
}

/* One Viterbi run over x[0..T) (quantize.py:218-320).
 *   overlap  < 0: free boundary; >= 0 pins s_0 >> K == overlap and
 *                 s_{T-1} & (S_PRE-1) == overlap.
 *   back_from < 0: full traceback into states[0..T);
 *            >= 0: returns the state at step back_from (links are only needed
 *                  for steps > back_from, quantize.py:273-277, 305-312). */
static int64_t viterbi_one(const float *x, int T, const float *lut, int K,
                           int L, int64_t overlap, int back_from,
                           int32_t *states, vit_ws *w) {
    const int64_t S = (int64_t)1 << L, NC = (int64_t)1 << K;
    const int64_t SP = (int64_t)1 << (L - K);
    const float INF = INFINITY;
    float *cost = w->cost, *best = w->best;
    uint16_t *bp = w->bp;

    for (int64_t s = 0; s < S; ++s) cost[s] = emit_sq(lut[s], x[0]);
    if (overlap >= 0) {           /* quantize.py:265-270: cost + mask */
        for (int64_t s = 0; s < S; ++s) {
            float m = ((s >> K) == overlap) ? 0.0f : INF;
            cost[s] = cost[s] + m;
        }
    }
    for (int i = 1; i < T; ++i) {
        for (int64_t j = 0; j < SP; ++j) {   /* cost.view(NC, S_PRE).min(0) */
            float bv = cost[j];
            int bi = 0;
            for (int64_t wv = 1; wv < NC; ++wv) {
                float c = cost[j + wv * SP];
                if (c < bv) { bv = c; bi = (int)wv; }
            }
            best[j] = bv;
            bp[(size_t)i * SP + j] = (uint16_t)bi;
        }
        const float xi = x[i];
        for (int64_t s = 0; s < S; ++s)      /* e.view(S_PRE, NC) += best */
            cost[s] = emit_sq(lut[s], xi) + best[s >> K];
    }
    if (overlap >= 0) {           /* quantize.py:298-303 */
        for (int64_t s = 0; s < S; ++s) {
            float m = ((s & (SP - 1)) == overlap) ? 0.0f : INF;
            cost[s] = cost[s] + m;
        }
    }
    int64_t sb = 0;               /* argmin, first index on ties */
    float cb = cost[0];
    for (int64_t s = 1; s < S; ++s)
        if (cost[s] < cb) { cb = cost[s]; sb = s; }

    int stop = back_from >= 0 ? back_from : 0;
    int64_t s = sb;
    if (states && back_from < 0) states[T - 1] = (int32_t)s;
    for (int i = T - 1; i > stop; --i) {      /* quantize.py:314-320 */
        int64_t j = s >> K;
        int64_t wv = bp[(size_t)i * SP + j];
        s = j + wv * SP;
        if (states && back_from < 0) states[i - 1] = (int32_t)s;
    }
    return s;
}

/* Exported: plain Viterbi on nseq sequences (X [nseq][T], states [nseq][T]).
 * overlaps may be NULL (free boundary).  Returns 0 or -1 on allocation
 * failure. */
int oracle_viterbi(const float *X, int nseq, int T, const float *lut, int K,
                   int L, const int64_t *overlaps, int32_t *states) {
    vit_ws w;
    if (ws_alloc(&w, L, K, T)) { ws_free(&w); return -1; }
    for (int b = 0; b < nseq; ++b)
        viterbi_one(X + (size_t)b * T, T, lut, K, L,
                    overlaps ? overlaps[b] : -1, -1,
                    states + (size_t)b * T, &w);
    ws_free(&w);
    return 0;
}

/* Exported: viterbi(..., back_from=bf) -> state at step bf for each seq. */
int oracle_viterbi_back_from(const float *X, int nseq, int T, const float *lut,
                             int K, int L, int back_from, int64_t *out) {
    vit_ws w;
    if (ws_alloc(&w, L, K, T)) { ws_free(&w); return -1; }
    for (int b = 0; b < nseq; ++b)
        out[b] = viterbi_one(X + (size_t)b * T, T, lut, K, L, -1, back_from,
                             NULL, &w);
    ws_free(&w);
    return 0;
}

/* quantize_seq_tailbite for one sequence (quantize.py:323-354). */
static void tailbite_one(const float *x, int T, const float *lut, int K,
                         int L, int pivot, int margin, int32_t *states,
                         float *roll, vit_ws *w) {
    for (int i = 0; i < T; ++i) {         /* torch.roll(X, pivot, 0) */
        int src = i - pivot;
        if (src < 0) src += T;
        roll[i] = x[src];
    }
    int64_t s_p;
    if (margin && pivot + margin < T)
        s_p = viterbi_one(roll, pivot + margin, lut, K, L, -1, pivot, NULL, w);
    else
        s_p = viterbi_one(roll, T, lut, K, L, -1, pivot, NULL, w);
    int64_t overlap = s_p >> K;
    viterbi_one(x, T, lut, K, L, overlap, -1, states, w);
}

typedef struct {
    const float *X;
    int nseq, T, K, L, pivot, margin;
    const float *lut;
    int32_t *states;
    int next;                 /* shared work counter */
    pthread_mutex_t mu;
    int err;
} tb_job;

static void *tb_worker(void *arg) {
    tb_job *jb = (tb_job *)arg;
    vit_ws w;
    float *roll = (float *)malloc((size_t)jb->T * sizeof(float));
    if (ws_alloc(&w, jb->L, jb->K, jb->T) || !roll) {
        pthread_mutex_lock(&jb->mu);
        jb->err = -1;
        pthread_mutex_unlock(&jb->mu);
        ws_free(&w);
        free(roll);
        return NULL;
    }
    for (;;) {
        pthread_mutex_lock(&jb->mu);
        int b = jb->next++;
        pthread_mutex_unlock(&jb->mu);
        if (b >= jb->nseq) break;
        tailbite_one(jb->X + (size_t)b * jb->T, jb->T, jb->lut, jb->K, jb->L,
                     jb->pivot, jb->margin, jb->states + (size_t)b * jb->T,
                     roll, &w);
    }
    ws_free(&w);
    free(roll);
    return NULL;
}

/* Exported: tail-biting encode of nseq sequences on nthreads host threads.
 * X [nseq][T] fp32, states [nseq][T] int32 (full L-bit states). */
int oracle_tailbite(const float *X, int nseq, int T, const float *lut, int K,
                    int L, int pivot, int margin, int nthreads,
                    int32_t *states) {
    if (pivot < 0 || pivot >= T || K < 1 || K >= L) return -2;
    tb_job jb = {X, nseq, T, K, L, pivot, margin, lut, states, 0,
                 PTHREAD_MUTEX_INITIALIZER, 0};
    if (nthreads < 1) nthreads = 1;
    if (nthreads > nseq) nthreads = nseq > 0 ? nseq : 1;
    pthread_t *th = (pthread_t *)malloc(sizeof(pthread_t) * (size_t)nthreads);
    if (!th) return -1;
    for (int t = 0; t < nthreads; ++t)
        pthread_create(&th[t], NULL, tb_worker, &jb);
    for (int t = 0; t < nthreads; ++t) pthread_join(th[t], NULL);
    free(th);
    return jb.err;
}
