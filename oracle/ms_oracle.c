/*
 * ORACLE — test infrastructure only.  Nothing in the product links this file;
 * only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load it,
 * as the checker.
 *
 * A plain-C restatement of mini.js's token sampler, src/generation.js:9-81,
 * that keeps the reference's JavaScript arithmetic:
 *   - every JS Number is an IEEE double, every Float32Array store rounds to
 *     fp32 (round to nearest even) and every load widens back to double;
 *   - `Math.exp` is V8's: a port of fdlibm's e_exp.c (V8 src/base/ieee754.cc,
 *     `ieee754::exp`), restated below as js_exp from the published fdlibm
 *     method (argument reduction by k*ln2 split in two parts, a degree-5
 *     Remez rational form on |r| <= 0.5*ln2, scaling by 2^k).  The C
 *     library's exp can be selected instead (msref_set_exp) to count where
 *     the two differ;
 *   - `idx.sort((a,b) => probs[b]-probs[a])` is a stable sort (Node >= 18), so
 *     the order is (prob desc, index asc); a comparator that returns NaN counts
 *     as "equal", which leaves an all-NaN row in index order;
 *   - sums run sequentially in index / candidate order.
 *
 * Parity status: pinned to the reference's arithmetic, not to a run of the
 * reference.  The reference's own tests pin no sampled id or probability
 * (greedy determinism and onToken counts only), and neither this machine nor
 * the GPU machines have a JavaScript engine to run src/generation.js itself.
 * The pins are: the known-answer cases in tests/golden/ (derived by hand from
 * the JS source text), and js_exp checked bit for bit against a second,
 * independent restatement of fdlibm's exp (tests/golden/fdlibm_exp.py) over
 * millions of arguments, and against the C library's exp within one ulp.
 *
 * Build: oracle/Makefile (gcc, -ffp-contract=off so no FMA changes a rounding).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "../include/minisample.h"

/* ------------------------------------------------------------------------ */
/* mulberry32 — test/synth.mjs:10-17 and src/selftest.js:10-18               */
/* ------------------------------------------------------------------------ */

uint32_t msref_mulberry32_u32(uint32_t* state) {
    uint32_t a = *state + 0x6d2b79f5u;               /* a = (a + 0x6d2b79f5) | 0 */
    *state = a;
    uint32_t t = (a ^ (a >> 15)) * (1u | a);          /* Math.imul(a ^ a>>>15, 1|a) */
    t = (t + (t ^ (t >> 7)) * (61u | t)) ^ t;         /* (t + imul(t ^ t>>>7, 61|t)) ^ t */
    return t ^ (t >> 14);                             /* (t ^ t>>>14) >>> 0 */
}

double msref_mulberry32(uint32_t* state) {
    return (double)msref_mulberry32_u32(state) / 4294967296.0;
}

/* ------------------------------------------------------------------------ */
/* Math.exp: fdlibm e_exp.c, as V8 ports it (src/base/ieee754.cc)            */
/* ------------------------------------------------------------------------ */
/*
 * exp(x) = 2^k * exp(r) with x = k*ln2 + r, |r| <= 0.5*ln2; ln2 is split into
 * a high part with trailing zero bits (so k*ln2_hi is exact) and a low part.
 * On the reduced range, R(r^2) = r*(e^r + 1)/(e^r - 1) ~ 2 + P1 z + ... + P5 z^5
 * (z = r^2, Remez coefficients published with fdlibm), and
 *   exp(r) = 1 + r + r*c/(2 - c),  c = r - z*(P1 + z*(P2 + ... + z*P5)).
 * Every operation below is one IEEE double operation (the oracle builds with
 * -ffp-contract=off), in fdlibm's order.
 */
static double bits_to_double(uint64_t b) { double d; memcpy(&d, &b, 8); return d; }
static uint64_t double_to_bits(double d) { uint64_t b; memcpy(&b, &d, 8); return b; }

static double js_exp(double x) {
    static const double ln2_hi[2] = {6.93147180369123816490e-01, -6.93147180369123816490e-01};
    static const double ln2_lo[2] = {1.90821492927058770002e-10, -1.90821492927058770002e-10};
    static const double half[2] = {0.5, -0.5};
    const double inv_ln2 = 1.44269504088896338700e+00;
    const double p1 = 1.66666666666666019037e-01, p2 = -2.77777777770155933842e-03,
                 p3 = 6.61375632143793436117e-05, p4 = -1.65339022054652515390e-06,
                 p5 = 4.13813679705723846039e-08;
    const double over = 7.09782712893383973096e+02, under = -7.45133219101941108420e+02;
    const double e_const = 2.718281828459045;
    const double two_m1000 = 9.33263618503218878990e-302; /* 2^-1000 */
    const uint64_t bx = double_to_bits(x);
    const uint32_t hi_word = (uint32_t)(bx >> 32);
    const int sign = (int)(hi_word >> 31);
    const uint32_t ahi = hi_word & 0x7fffffffu;

    if (ahi >= 0x40862E42u) {                        /* |x| >= 709.78 or not finite */
        if (ahi >= 0x7ff00000u) {
            if (((ahi & 0xfffffu) | (uint32_t)bx) != 0) return x + x;   /* NaN */
            return sign ? 0.0 : x;                                     /* exp(-inf)=0, exp(inf)=inf */
        }
        if (x > over) return INFINITY;
        if (x < under) return 0.0;
    }
    double hi = 0.0, lo = 0.0, r;
    int k = 0;
    if (ahi > 0x3FD62E42u) {                         /* |x| > 0.5 ln2 */
        if (ahi < 0x3FF0A2B2u) {                     /* and |x| < 1.5 ln2: k = +-1 */
            if (x == 1.0) return e_const;            /* V8 returns E exactly here */
            hi = x - ln2_hi[sign];
            lo = ln2_lo[sign];
            k = 1 - sign - sign;
        } else {
            k = (int)(inv_ln2 * x + half[sign]);
            const double t = (double)k;
            hi = x - t * ln2_hi[0];                  /* exact: ln2_hi has trailing zeros */
            lo = t * ln2_lo[0];
        }
        r = hi - lo;
    } else if (ahi < 0x3e300000u) {                  /* |x| < 2^-28 */
        return 1.0 + x;
    } else {
        r = x;
    }
    const double z = r * r;
    const double c = r - z * (p1 + z * (p2 + z * (p3 + z * (p4 + z * p5))));
    if (k == 0) return 1.0 - ((r * c) / (c - 2.0) - r);
    const double y = 1.0 - ((lo - (r * c) / (2.0 - c)) - hi);
    /* scale by 2^k: exact exponent arithmetic while the result stays normal */
    if (k >= -1021) {
        if (k == 1024) return y * 2.0 * bits_to_double(0x7fe0000000000000ull);
        return y * bits_to_double((uint64_t)(0x3ff + k) << 52);
    }
    return y * bits_to_double((uint64_t)(0x3ff + k + 1000) << 52) * two_m1000;
}

static int g_use_libc_exp = 0;

/* 0: Math.exp as V8 computes it (js_exp, the default); 1: the C library's exp. */
void msref_set_exp(int use_libc) { g_use_libc_exp = use_libc ? 1 : 0; }

double msref_exp(double x) { return g_use_libc_exp ? exp(x) : js_exp(x); }

/* The fp32 softmax term fp32(exp(x - mx)) of src/generation.js:14, with V8's
 * exp and with the C library's, for counting where they differ. */
void msref_terms_both(const float* xs, int64_t n, double mx, float* t_js, float* t_libc) {
    for (int64_t i = 0; i < n; i++) {
        const double d = (double)xs[i] - mx;
        if (t_js) t_js[i] = (float)js_exp(d);
        if (t_libc) t_libc[i] = (float)exp(d);
    }
}

/* ------------------------------------------------------------------------ */
/* Per-row diagnostics                                                      */
/* ------------------------------------------------------------------------ */

typedef struct msref_row_diag {
    double  mx;          /* softmaxTopNothing's mx (max of the tempered row)      */
    double  sum;         /* softmaxTopNothing's sum                               */
    int32_t greedy;      /* 1 when argmax was taken                              */
    int32_t nan_path;    /* 1 when the probabilities are NaN                     */
    int64_t n_topk;      /* candidates after the top-k slice                     */
    int64_t n_cand;      /* candidates after the top-p slice                     */
    double  total;       /* fp64 sum of the candidate probabilities              */
    double  r;           /* Math.random() * total                                */
    int64_t draw_pos;    /* position in cand of the drawn id (-1 greedy)          */
    double  margin_draw; /* distance of r from the nearest cumulative boundary    */
    double  margin_cut;  /* distance of topP from the nearest running acc value   */
    int32_t cand_cap;    /* capacity of cand_ids / cand_probs                     */
    int32_t* cand_ids;   /* first min(n_cand, cand_cap) candidates               */
    float*  cand_probs;
} msref_row_diag;

typedef struct {
    float p;
    int32_t i;
} prob_idx;

static int cmp_prob_desc_idx_asc(const void* a, const void* b) {
    const prob_idx* x = (const prob_idx*)a;
    const prob_idx* y = (const prob_idx*)b;
    if (x->p > y->p) return -1;
    if (x->p < y->p) return 1;
    return (x->i > y->i) - (x->i < y->i);
}

/* argmax — src/generation.js:51-55: first index of the strict maximum. */
static int64_t ref_argmax(const float* w, int64_t V) {
    int64_t best = 0;
    for (int64_t i = 1; i < V; i++)
        if ((double)w[i] > (double)w[best]) best = i;
    return best;
}

/*
 * applyRepetitionPenalty — src/generation.js:19-25.  `new Set(ids)` visits each
 * distinct id once; a typed-array access outside [0, V) reads undefined and the
 * store is dropped, so such ids change nothing.  `seen` is scratch of V bytes.
 */
static void ref_penalty(float* w, int64_t V, const int32_t* hist, int64_t H, double pen,
                        unsigned char* seen) {
    memset(seen, 0, (size_t)V);
    for (int64_t h = 0; h < H; h++) {
        int64_t id = hist[h];
        if (id < 0 || id >= V || seen[id]) continue;
        seen[id] = 1;
        double v = (double)w[id];
        w[id] = (float)(v > 0 ? v / pen : v * pen);
    }
}

/*
 * pickToken — src/generation.js:71-81 with softmaxTopNothing (:9-17) and
 * sampleTopKTopP (:27-49) inlined.  `work` and `probs` are scratch of V floats,
 * `pairs` scratch of V prob_idx, `seen` scratch of V bytes.  Returns the id.
 */
static int32_t ref_pick(const float* logits, int64_t V, const int32_t* hist, int64_t H,
                        const ms_params* p, double u, msref_row_diag* d, float* work,
                        float* probs, prob_idx* pairs, unsigned char* seen, float* pen_out) {
    /* :72  work = Float32Array.from(lastLogits) */
    memcpy(work, logits, (size_t)V * sizeof(float));
    msref_row_diag dd;
    memset(&dd, 0, sizeof dd);
    dd.draw_pos = -1;
    dd.margin_draw = INFINITY;
    dd.margin_cut = INFINITY;

    /* :73-75  penalty iff opts.repetitionPenalty truthy, !== 1.0, generated.length */
    double pen = p->repetition_penalty;
    if (pen != 0 && !isnan(pen) && pen != 1.0 && H > 0) ref_penalty(work, V, hist, H, pen, seen);
    if (pen_out) memcpy(pen_out, work, (size_t)V * sizeof(float));

    /* :76  greedy */
    double T = p->temperature;
    if (!p->do_sample || T <= 0.0001) {
        dd.greedy = 1;
        int32_t id = (int32_t)ref_argmax(work, V);
        if (d) {
            int32_t cap = d->cand_cap; int32_t* ci = d->cand_ids; float* cp = d->cand_probs;
            *d = dd; d->cand_cap = cap; d->cand_ids = ci; d->cand_probs = cp;
        }
        return id;
    }
    /* :77-79  temperature */
    if (T != 1.0)
        for (int64_t i = 0; i < V; i++) work[i] = (float)((double)work[i] / T);

    /* :9-17  softmaxTopNothing */
    double mx = -INFINITY;
    for (int64_t i = 0; i < V; i++)
        if ((double)work[i] > mx) mx = (double)work[i];
    double sum = 0;
    for (int64_t i = 0; i < V; i++) {
        probs[i] = (float)msref_exp((double)work[i] - mx);
        sum += (double)probs[i];
    }
    for (int64_t i = 0; i < V; i++) probs[i] = (float)((double)probs[i] / sum);
    dd.mx = mx;
    dd.sum = sum;
    dd.nan_path = isnan(sum) ? 1 : 0;

    /* :28-30  idx sorted by prob desc, stable */
    for (int64_t i = 0; i < V; i++) { pairs[i].p = probs[i]; pairs[i].i = (int32_t)i; }
    if (!dd.nan_path) qsort(pairs, (size_t)V, sizeof(prob_idx), cmp_prob_desc_idx_asc);

    /* :31-32  top-k */
    int64_t n = V;
    int32_t K = p->top_k;
    if (K != 0 && K > 0 && K < V) n = K;
    dd.n_topk = n;

    /* :33-40  top-p */
    double P = p->top_p;
    if (P != 0 && P < 1) {
        double acc = 0, prev = 0;
        int64_t cut = n;
        for (int64_t i = 0; i < n; i++) {
            prev = acc;
            acc += (double)pairs[i].p;
            if (acc >= P) { cut = i + 1; break; }
        }
        if (cut < n || acc >= P) {
            double m = acc - P;
            if (cut > 1 && P - prev < m) m = P - prev;
            dd.margin_cut = m;
        } else {
            dd.margin_cut = P - acc;
        }
        n = cut > 1 ? cut : 1;
    }
    dd.n_cand = n;

    /* :41-48  draw */
    double total = 0;
    for (int64_t i = 0; i < n; i++) total += (double)pairs[i].p;
    double r = u * total;
    dd.total = total;
    dd.r = r;
    int32_t id = pairs[n - 1].i;
    dd.draw_pos = n - 1;
    double rr = r;
    for (int64_t i = 0; i < n; i++) {
        double before = rr;
        rr -= (double)pairs[i].p;
        if (rr <= 0) {
            id = pairs[i].i;
            dd.draw_pos = i;
            dd.margin_draw = fmin(before, -rr);
            break;
        }
    }
    if (rr > 0) dd.margin_draw = rr;
    if (d) {
        int32_t cap = d->cand_cap; int32_t* ci = d->cand_ids; float* cp = d->cand_probs;
        *d = dd; d->cand_cap = cap; d->cand_ids = ci; d->cand_probs = cp;
        for (int64_t i = 0; i < n && i < cap; i++) {
            if (ci) ci[i] = pairs[i].i;
            if (cp) cp[i] = pairs[i].p;
        }
    }
    return id;
}

/* ------------------------------------------------------------------------ */
/* Public entry points                                                      */
/* ------------------------------------------------------------------------ */

/*
 * One row.  work_out / probs_out (nullable, [V]) receive the reference's
 * `work` array as handed to argmax / softmax and the softmax output.
 */
int32_t msref_pick_token(const float* logits, int64_t V, const int32_t* hist, int64_t H,
                         const ms_params* p, double u, msref_row_diag* d, float* work_out,
                         float* probs_out) {
    float* work = (float*)malloc((size_t)V * sizeof(float));
    float* probs = (float*)malloc((size_t)V * sizeof(float));
    prob_idx* pairs = (prob_idx*)malloc((size_t)V * sizeof(prob_idx));
    unsigned char* seen = (unsigned char*)malloc((size_t)V);
    if (!work || !probs || !pairs || !seen) {
        free(work); free(probs); free(pairs); free(seen);
        return -1;
    }
    int32_t id = ref_pick(logits, V, hist, H, p, u, d, work, probs, pairs, seen, NULL);
    if (work_out) memcpy(work_out, work, (size_t)V * sizeof(float));
    if (probs_out) memcpy(probs_out, probs, (size_t)V * sizeof(float));
    free(work); free(probs); free(pairs); free(seen);
    return id;
}

typedef struct {
    const float* logits; int64_t B, V, ld;
    const int32_t* hist; const int64_t* hist_off;
    const ms_params* p; const double* u; int32_t* out;
    msref_row_diag* diags;
    float* pen_out; /* [B, V] or NULL */
    int64_t next;   /* shared row counter */
    pthread_mutex_t mu;
    int err;
} batch_job;

static void* batch_worker(void* arg) {
    batch_job* j = (batch_job*)arg;
    int64_t V = j->V;
    float* work = (float*)malloc((size_t)V * sizeof(float));
    float* probs = (float*)malloc((size_t)V * sizeof(float));
    prob_idx* pairs = (prob_idx*)malloc((size_t)V * sizeof(prob_idx));
    unsigned char* seen = (unsigned char*)malloc((size_t)V);
    if (!work || !probs || !pairs || !seen) {
        pthread_mutex_lock(&j->mu); j->err = -1; pthread_mutex_unlock(&j->mu);
    } else {
        for (;;) {
            pthread_mutex_lock(&j->mu);
            int64_t r = j->next++;
            pthread_mutex_unlock(&j->mu);
            if (r >= j->B) break;
            const int32_t* h = NULL;
            int64_t H = 0;
            if (j->hist_off && j->hist) {
                h = j->hist + j->hist_off[r];
                H = j->hist_off[r + 1] - j->hist_off[r];
            }
            double u = j->u ? j->u[r] : 0.0;
            j->out[r] = ref_pick(j->logits + r * j->ld, V, h, H, j->p, u,
                                 j->diags ? &j->diags[r] : NULL, work, probs, pairs, seen,
                                 j->pen_out ? j->pen_out + r * V : NULL);
        }
    }
    free(work); free(probs); free(pairs); free(seen);
    return NULL;
}

/*
 * B rows, each exactly as pickToken (no batching exists in the reference, so
 * a batch is B independent calls).  Rows are spread over `nthreads` threads.
 * pen_out (nullable, [B, V]) receives each row's `work` after the penalty
 * (src/generation.js:72-75).
 */
int msref_sample_batch(const float* logits, int64_t B, int64_t V, int64_t ld,
                       const int32_t* hist, const int64_t* hist_off, const ms_params* p,
                       const double* u, int32_t* out_ids, msref_row_diag* diags,
                       int nthreads, float* pen_out) {
    if (B < 0 || V < 1 || ld < V || !logits || !p || !out_ids) return -1;
    batch_job j;
    memset(&j, 0, sizeof j);
    j.logits = logits; j.B = B; j.V = V; j.ld = ld; j.hist = hist; j.hist_off = hist_off;
    j.p = p; j.u = u; j.out = out_ids; j.diags = diags; j.next = 0; j.pen_out = pen_out;
    pthread_mutex_init(&j.mu, NULL);
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    pthread_t th[256];
    int started = 0;
    for (int t = 1; t < nthreads; t++)
        if (pthread_create(&th[started], NULL, batch_worker, &j) == 0) started++;
    batch_worker(&j);
    for (int t = 0; t < started; t++) pthread_join(th[t], NULL);
    pthread_mutex_destroy(&j.mu);
    return j.err;
}

int msref_row_diag_size(void) { return (int)sizeof(msref_row_diag); }
