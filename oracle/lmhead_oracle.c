/* CPU oracle of the output projection (LM head) of a MiniMax layer stack — TEST INFRASTRUCTURE ONLY.
 *
 * Restates, in plain C, the reference's end of a decode step (src/tensor_parallel_model.rs:871-880:
 * output_norm, then the Q6_K `output` QMatMul, then greedy sampling, src/sampling.rs:84-88):
 *   the GGUF Q6_K block (210 bytes per 256 weights: ql[128] low 4 bits, qh[64] high 2 bits, int8
 *   scales[16], half d) and its dequantisation (dequantize_block_q6_K, quantized.cu:1025-1050),
 *   the Q6_K x Q8_1 matvec (vec_dot_q6_K_q8_1, mmvq_gguf.cu:384-400, 609-632; the activation
 *   quantised by quantize_q8_1),
 *   the greedy choice: the first index of the maximum logit.
 * The matvec is exact up to its final rounding: every term d * sc * d8 * sum(q6 q8) is a product
 * of two halves, an int8 and an integer of at most 17 bits, exact in double, and the terms are
 * summed in double.
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU baseline use this file.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "moe_oracle.h"

/* Signed 6-bit value (q - 32) of element e (0-255) of a Q6_K block. */
static int q6k_value(const uint8_t *blk, int e) {
    const uint8_t *ql = blk, *qh = blk + 128;
    const int half = e / 128, r = e % 128, quarter = r / 32, l = r % 32;
    const uint8_t lo = ql[64 * half + l + (quarter & 1) * 32];
    const int low4 = (quarter < 2) ? (lo & 0xF) : (lo >> 4);
    const int high2 = (qh[32 * half + l] >> (2 * quarter)) & 3;
    return (low4 | (high2 << 4)) - 32;
}

/* Scale index (0-15) of element e: 16 consecutive elements share one int8 scale. */
static int q6k_scale_index(int e) { return e / 16; }

void orc_q6k_dequant_row(const uint8_t *row, int k, float *out) {
    for (int b = 0; b < k / 256; ++b) {
        const uint8_t *blk = row + (size_t)b * 210;
        uint16_t dh;
        memcpy(&dh, blk + 208, 2);
        const float d = orc_half_to_float(dh);
        for (int e = 0; e < 256; ++e) {
            const int sc = (int8_t)blk[192 + q6k_scale_index(e)];
            out[b * 256 + e] = d * (float)sc * (float)q6k_value(blk, e);
        }
    }
}

/* y[r] = sum over 16-element groups of d * sc * d8(block) * sum(q6 * q8), x quantised to Q8_1. */
void orc_q6k_matvec(const uint8_t *w, int rows, int k, const float *x, float *y) {
    const int nsb = k / 256, nb = k / 32;
    uint8_t *xq = (uint8_t *)malloc((size_t)36 * nb);
    orc_quantize_q8_1(x, 1, k, k, xq);
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r) {
        const uint8_t *row = w + (size_t)r * nsb * 210;
        double acc = 0.0;
        for (int b = 0; b < nsb; ++b) {
            const uint8_t *blk = row + (size_t)b * 210;
            uint16_t dh;
            memcpy(&dh, blk + 208, 2);
            const double d = orc_half_to_float(dh);
            for (int g = 0; g < 16; ++g) {
                const int e0 = 16 * g;
                const uint8_t *xb = xq + (size_t)(b * 8 + e0 / 32) * 36;
                uint16_t d8h;
                memcpy(&d8h, xb, 2);
                int32_t isum = 0;
                for (int j = 0; j < 16; ++j)
                    isum += q6k_value(blk, e0 + j) * (int32_t)(int8_t)xb[4 + (e0 + j) % 32];
                acc += d * (double)(int8_t)blk[192 + g] * (double)orc_half_to_float(d8h) * (double)isum;
            }
        }
        y[r] = (float)acc;
    }
    free(xq);
}

/* First index of the maximum (NaN never compares greater); -1 for n <= 0. */
int orc_argmax_f32(const float *v, int n) {
    int best = -1;
    for (int i = 0; i < n; ++i)
        if (!isnan(v[i]) && (best < 0 || v[i] > v[best])) best = i;
    return best;
}
