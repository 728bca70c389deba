/* CPU oracle of the decode-attention half of a MiniMax layer — TEST INFRASTRUCTURE ONLY.
 *
 * Restates, in plain C, the reference's single-token attention path:
 *   Q8_0 x Q8_1 matvec of Q / K / V and of the output projection (mmvq_gguf.cu:282-290, 477-490,
 *   814-836; the activation quantised by quantize_q8_1, mmvq_gguf.cu:1137-1169),
 *   RMSNorm of Q and K with f16 output (mmvq_gguf.cu:838-885),
 *   partial rotary embedding on f16 (mmvq_gguf.cu:1038-1066),
 *   split-K GQA decode attention with its combine (decode_attention.cu:311-843).
 * The matvecs are exact up to the final rounding (every term sumi * d_w * d_x is a 42-bit
 * integer multiple of a power of two, summed in double); the rotary embedding reproduces the
 * reference's half-precision operations bit for bit; RMSNorm and softmax run in double.
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU baseline use this file.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "moe_oracle.h"

/* IEEE binary16 of a double, round to nearest even (the sum of two halves is exact in double,
 * so a half add / subtract is this of the exact sum). */
uint16_t orc_double_to_half(double v) {
    const uint16_t sign = signbit(v) ? 0x8000u : 0u;
    const double a = fabs(v);
    if (isnan(v)) return 0x7E00u;
    if (a >= 65520.0) return sign | 0x7C00u;
    if (a < 6.103515625e-05) return sign | (uint16_t)nearbyint(a * 16777216.0); /* subnormal, 2^-24 units */
    int e;
    const double f = frexp(a, &e); /* a = f * 2^e, f in [0.5, 1) */
    double m = nearbyint(f * 2048.0);
    if (m == 2048.0) {
        m = 1024.0;
        ++e;
    }
    const int he = e + 14;
    if (he >= 31) return sign | 0x7C00u;
    return sign | (uint16_t)(he << 10) | (uint16_t)(m - 1024.0);
}

static uint16_t h_mul(uint16_t a, uint16_t b) {
    return orc_double_to_half((double)orc_half_to_float(a) * (double)orc_half_to_float(b));
}
/* half fma: a * b + c rounded once (a product of halves is exact in double, and so is its sum
 * with a half) */
static uint16_t h_fma(uint16_t a, uint16_t b, double c) {
    return orc_double_to_half((double)orc_half_to_float(a) * (double)orc_half_to_float(b) + c);
}

/* y[r] = sum over 32-blocks b of sumi(r, b) * d_w(r, b) * d_x(b), x quantised to Q8_1
 * (d_x = half(amax / 127)).  w: rows x (k / 32) blocks of 34 bytes (half d, 32 int8). */
void orc_q8_0_matvec(const uint8_t *w, int rows, int k, const float *x, float *y) {
    const int nb = k / 32;
    uint8_t *xq = (uint8_t *)malloc((size_t)36 * nb);
    orc_quantize_q8_1(x, 1, k, k, xq);
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r) {
        const uint8_t *row = w + (size_t)r * nb * 34;
        double acc = 0.0;
        for (int b = 0; b < nb; ++b) {
            const uint8_t *blk = row + (size_t)b * 34, *xb = xq + (size_t)b * 36;
            uint16_t dw, dx;
            memcpy(&dw, blk, 2);
            memcpy(&dx, xb, 2);
            int32_t sumi = 0;
            for (int i = 0; i < 32; ++i) sumi += (int32_t)(int8_t)blk[2 + i] * (int32_t)(int8_t)xb[4 + i];
            acc += (double)sumi * (double)orc_half_to_float(dw) * (double)orc_half_to_float(dx);
        }
        y[r] = (float)acc;
    }
    free(xq);
}

/* dst (f16): Q and K rows scaled by 1 / sqrt(mean(v^2) + eps) and their norm weights, V copied. */
void orc_qkv_rmsnorm_f16(const float *proj, const float *q_alpha, const float *k_alpha, int q_rows,
                         int k_rows, int v_rows, float eps, uint16_t *dst) {
    for (int p = 0; p < 3; ++p) {
        const int n = p == 0 ? q_rows : (p == 1 ? k_rows : v_rows);
        const int off = p == 0 ? 0 : (p == 1 ? q_rows : q_rows + k_rows);
        if (p == 2) {
            for (int i = 0; i < n; ++i) dst[off + i] = orc_double_to_half(proj[off + i]);
            continue;
        }
        double ss = 0.0;
        for (int i = 0; i < n; ++i) ss += (double)proj[off + i] * proj[off + i];
        const double scale = 1.0 / sqrt(ss / n + (double)eps);
        const float *alpha = p == 0 ? q_alpha : k_alpha;
        for (int i = 0; i < n; ++i) dst[off + i] = orc_double_to_half(scale * proj[off + i] * alpha[i]);
    }
}

/* Partial rotary embedding: in every head_dim-wide head, the first rope_dim columns are rotated
 * in half precision, the rest copied; c / s are the f32 table entries rounded to half.  The
 * reference's `__hsub(__hmul(x, c), __hmul(x', s))` / `__hadd(__hmul(x', s), __hmul(x, c))`, as nvcc
 * compiles them with its default multiply-add contraction, compute fma(x, c, -rn(x' * s)) and
 * fma(x', s, rn(x * c)) in half (pinned bit for bit by the golden vectors).
 * dst = [Q rows | K rows]. */
void orc_partial_rope_f16(const uint16_t *q, const uint16_t *k, const float *cosv, const float *sinv, int q_rows,
                          int k_rows, int head_dim, int rope_dim, int position, uint16_t *dst) {
    const int half_rope = rope_dim / 2;
    for (int idx = 0; idx < q_rows + k_rows; ++idx) {
        const int is_q = idx < q_rows;
        const int local = is_q ? idx : idx - q_rows;
        const uint16_t *src = is_q ? q : k;
        const int col = local % head_dim;
        if (col >= rope_dim) {
            dst[idx] = src[local];
            continue;
        }
        const int pair = col < half_rope ? local + half_rope : local - half_rope;
        const int freq = col < half_rope ? col : col - half_rope;
        const uint16_t c = orc_float_to_half(cosv[position * half_rope + freq]);
        const uint16_t s = orc_float_to_half(sinv[position * half_rope + freq]);
        dst[idx] = col < half_rope ? h_fma(src[local], c, -(double)orc_half_to_float(h_mul(src[pair], s)))
                                   : h_fma(src[pair], s, (double)orc_half_to_float(h_mul(src[local], c)));
    }
}

/* Single-token GQA: query head h attends to KV head h / (q_heads / kv_heads) over positions
 * [0, seq_len); K / V of head g, position t at k + g * kv_head_stride + t * head_dim (f16).
 * out [q_heads][head_dim] f16 = softmax(scale * q.k) . v, in double. */
void orc_gqa_decode_f16(const uint16_t *q, const uint16_t *k, const uint16_t *v, int seq_len, int q_heads,
                        int kv_heads, int head_dim, int64_t kv_head_stride, float scale, uint16_t *out) {
    const int group = q_heads / kv_heads;
#pragma omp parallel for schedule(static)
    for (int h = 0; h < q_heads; ++h) {
        const uint16_t *kh = k + (int64_t)(h / group) * kv_head_stride;
        const uint16_t *vh = v + (int64_t)(h / group) * kv_head_stride;
        double *s = (double *)malloc(sizeof(double) * (size_t)(seq_len > 0 ? seq_len : 1));
        double mx = -INFINITY;
        for (int t = 0; t < seq_len; ++t) {
            double dot = 0.0;
            for (int d = 0; d < head_dim; ++d)
                dot += (double)orc_half_to_float(q[h * head_dim + d]) * orc_half_to_float(kh[(int64_t)t * head_dim + d]);
            s[t] = dot * scale;
            if (s[t] > mx) mx = s[t];
        }
        double den = 0.0;
        for (int t = 0; t < seq_len; ++t) {
            s[t] = exp(s[t] - mx);
            den += s[t];
        }
        for (int d = 0; d < head_dim; ++d) {
            double a = 0.0;
            for (int t = 0; t < seq_len; ++t) a += s[t] * orc_half_to_float(vh[(int64_t)t * head_dim + d]);
            out[h * head_dim + d] = orc_double_to_half(a / den);
        }
        free(s);
    }
}
