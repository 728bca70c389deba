/* CPU oracle of token sampling — TEST INFRASTRUCTURE ONLY.
 *
 * Restates, in plain C, the reference's sampler (src/sampling.rs):
 *   SamplingParams::validate (:31-39): temperature finite and >= 0; top_p finite in [0, 1];
 *   TokenSampler::sample (:84-150): temperature 0 -> logits.argmax; otherwise non-finite logits
 *     are an error, candidates = (id, logit), cut to the top_k largest (compare_candidates,
 *     :154-159: logit descending by f32::total_cmp, then id ascending), then with top_p < 1 and
 *     more than one candidate: sorted, weights exp(l - max) (exponential_weights, :161-177, at
 *     temperature 1), kept up to and including the first whose running sum reaches
 *     top_p * sum; then weights exp((l - max) / temperature) over what is left, sample = u * total,
 *     walk: return the first candidate with sample < weight, else subtract its weight; the last
 *     candidate with a positive weight when the walk runs out;
 *   token_logprob (:60-75): ln softmax(logits)[id].
 * Weights and sums are double and summed in the reference's order; exp / log are the C library's
 * (the functions Rust's f64::exp / f64::ln call on Linux).
 * The one order the reference leaves to its standard library: with 0 < top_k < vocab and no top-p
 * cut, the walk visits the top_k candidates in the order select_nth_unstable_by left them; this
 * oracle (and the CUDA path) visits them by ascending id.  Without a top-k cut the reference's
 * order is ascending id too.
 * `margin` reports how close the call came to a different answer: the smallest gap, relative to
 * the sum it was compared against, between a compared value and its bound (top-p threshold,
 * sample vs weight).  A CUDA result may differ only when the margin is at rounding level.
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU baseline use this file.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "moe_oracle.h"

typedef struct {
    uint32_t id;
    float logit;
} orc_cand;

/* f32::total_cmp as an unsigned order. */
static uint32_t total_order(float v) {
    uint32_t u;
    memcpy(&u, &v, 4);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

static int cmp_cand(const void *a, const void *b) {
    const orc_cand *l = (const orc_cand *)a, *r = (const orc_cand *)b;
    const uint32_t ol = total_order(l->logit), orr = total_order(r->logit);
    if (ol != orr) return ol > orr ? -1 : 1; /* larger logit first */
    return l->id < r->id ? -1 : (l->id > r->id);
}

static int cmp_id(const void *a, const void *b) {
    const orc_cand *l = (const orc_cand *)a, *r = (const orc_cand *)b;
    return l->id < r->id ? -1 : (l->id > r->id);
}

static double rel_gap(double a, double b, double scale) {
    const double g = fabs(a - b);
    return scale > 0.0 ? g / scale : g;
}

int orc_sample_token(const float *logits, int vocab, double temperature, double top_p, int top_k, double u,
                     int32_t *token, double *margin) {
    *margin = INFINITY;
    if (!isfinite(temperature) || temperature < 0.0 || !isfinite(top_p) || top_p < 0.0 || top_p > 1.0)
        return MMRS_ERR_ARG_ORC;
    if (vocab < 1) return MMRS_ERR_ARG_ORC;
    if (temperature == 0.0) {
        *token = orc_argmax_f32(logits, vocab);
        return 0;
    }
    for (int i = 0; i < vocab; ++i)
        if (!isfinite(logits[i])) return MMRS_ERR_NONFINITE_ORC;
    orc_cand *c = (orc_cand *)malloc(sizeof(orc_cand) * (size_t)vocab);
    for (int i = 0; i < vocab; ++i) {
        c[i].id = (uint32_t)i;
        c[i].logit = logits[i];
    }
    size_t n = (size_t)vocab;
    const int sorted_cut = top_p < 1.0;
    if (top_k > 0 && (size_t)top_k < n) {
        qsort(c, n, sizeof(orc_cand), cmp_cand);
        n = (size_t)top_k;
        if (!(sorted_cut && n > 1)) qsort(c, n, sizeof(orc_cand), cmp_id); /* walk by ascending id */
    }
    if (sorted_cut && n > 1) {
        qsort(c, n, sizeof(orc_cand), cmp_cand);
        const double mx = (double)c[0].logit;
        double sum = 0.0;
        double *w = (double *)malloc(sizeof(double) * n);
        for (size_t i = 0; i < n; ++i) {
            w[i] = exp((double)c[i].logit - mx);
            sum += w[i];
        }
        const double threshold = sum * top_p;
        double cumulative = 0.0;
        size_t keep = n;
        for (size_t i = 0; i < n; ++i) {
            cumulative += w[i];
            const double g = rel_gap(cumulative, threshold, sum);
            if (g < *margin) *margin = g;
            if (cumulative >= threshold) {
                keep = i + 1;
                break;
            }
        }
        free(w);
        n = keep > 1 ? keep : 1;
    }
    double mx = -INFINITY;
    for (size_t i = 0; i < n; ++i)
        if ((double)c[i].logit > mx) mx = (double)c[i].logit;
    double *w = (double *)malloc(sizeof(double) * n);
    double total = 0.0;
    for (size_t i = 0; i < n; ++i) {
        w[i] = exp(((double)c[i].logit - mx) / temperature);
        total += w[i];
    }
    double sample = u * total;
    uint32_t fallback = c[0].id;
    int32_t pick = -1;
    for (size_t i = 0; i < n; ++i) {
        if (w[i] > 0.0) fallback = c[i].id;
        const double g = rel_gap(sample, w[i], total);
        if (w[i] > 0.0 && g < *margin) *margin = g;
        if (sample < w[i]) {
            pick = (int32_t)c[i].id;
            break;
        }
        sample -= w[i];
    }
    *token = pick >= 0 ? pick : (int32_t)fallback;
    free(w);
    free(c);
    return 0;
}

int orc_token_logprob(const float *logits, int vocab, int token_id, float *out) {
    if (token_id < 0 || token_id >= vocab) return MMRS_ERR_ARG_ORC;
    double mx = -INFINITY;
    int has_nan = 0;
    for (int i = 0; i < vocab; ++i) {
        if (logits[i] != logits[i]) has_nan = 1;
        if ((double)logits[i] > mx) mx = (double)logits[i];
    }
    double s = 0.0;
    for (int i = 0; i < vocab; ++i) s += exp((double)logits[i] - mx);
    const float v = has_nan ? NAN : (float)((double)logits[token_id] - mx - log(s));
    *out = v;
    return isfinite(v) ? 0 : MMRS_ERR_NONFINITE_ORC;
}
