/*
 * CPU oracle for the MiniMax-M2.7 sparse-MoE hot path — TEST INFRASTRUCTURE ONLY.
 *
 * Restates the reference's arithmetic (spmurrayzzz/minimax-rs, vendored Candle CUDA kernels)
 * in plain C so the CUDA product path can be checked against it and so a CPU baseline can be
 * timed.  Nothing in the product library links this file.  Build: see oracle/Makefile
 * (-O3 -ffp-contract=off -fopenmp; explicit fmaf() wherever the reference's compiled code fuses).
 *
 * Parity pins (tests/golden/README.md): dequant, Q8_1 bytes, routing and the decode / generic /
 * MMQ expert GEMMs are compared with the reference's own CUDA kernels compiled from the
 * reference sources (oracle/_ref) on seeded inputs; route sorting is pinned to the reference's
 * stable-grouping check (examples/moe_kernel_bench.rs:61-87); the all-reduce to the exact-sum
 * check of tests/tp_collective.rs:18-104.
 */
#include "moe_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define HOT __attribute__((target_clones("arch=x86-64-v3", "default")))

/* ------------------------------------------------------------------------------------ */
/* IEEE binary16 <-> binary32                                                            */
/* ------------------------------------------------------------------------------------ */
float orc_half_to_float(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t mant = h & 0x3ffu;
    uint32_t bits;
    if (exp == 0) {
        if (mant == 0) {
            bits = sign;
        } else { /* subnormal: renormalise */
            int e = -1;
            do {
                e++;
                mant <<= 1;
            } while ((mant & 0x400u) == 0);
            mant &= 0x3ffu;
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (mant << 13);
        }
    } else if (exp == 0x1f) {
        bits = sign | 0x7f800000u | (mant << 13);
    } else {
        bits = sign | ((exp - 15 + 127) << 23) | (mant << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

uint16_t orc_float_to_half(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t exp = (x >> 23) & 0xffu;
    uint32_t mant = x & 0x7fffffu;
    if (exp == 0xff) return (uint16_t)(sign | 0x7c00u | (mant ? (0x200u | (mant >> 13)) : 0));
    int e = (int)exp - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        mant |= 0x800000u;
        int shift = 14 - e;
        uint32_t hm = mant >> shift;
        uint32_t rem = mant & ((1u << shift) - 1u);
        uint32_t halfway = 1u << (shift - 1);
        if (rem > halfway || (rem == halfway && (hm & 1u))) hm++;
        return (uint16_t)(sign | hm);
    }
    uint32_t hm = mant >> 13;
    uint32_t rem = mant & 0x1fffu;
    uint32_t h = sign | ((uint32_t)e << 10) | hm;
    if (rem > 0x1000u || (rem == 0x1000u && (hm & 1u))) h++;
    return (uint16_t)h;
}

static inline float h2f(const uint8_t *p) {
    uint16_t h;
    memcpy(&h, p, 2);
    return orc_half_to_float(h);
}

size_t orc_row_bytes(int gguf_type, int k) {
    if (gguf_type == ORC_Q4K) return (size_t)(k / ORC_QK_K) * ORC_Q4K_BYTES;
    if (gguf_type == ORC_Q5K) return (size_t)(k / ORC_QK_K) * ORC_Q5K_BYTES;
    return 0;
}

static inline int pad_to(int v, int p) { return (v + p - 1) / p * p; }

int orc_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* Sets the OpenMP team size of the following calls (n <= 0: all hardware threads).  A launcher
 * such as torchrun exports OMP_NUM_THREADS=1 to its workers; a timed CPU baseline sets the team
 * size here instead of inheriting that. */
void orc_set_threads(int n) {
    omp_set_num_threads(n > 0 ? n : omp_get_num_procs());
}

/* ------------------------------------------------------------------------------------ */
/* k-quant super-block unpacking                                                         */
/* ------------------------------------------------------------------------------------ */
/* get_scale_min_k4 (quantized.cu:926-933): 8 six-bit scales and mins packed in 12 bytes. */
static inline void scale_min_k4(int j, const uint8_t *q, int *sc, int *m) {
    if (j < 4) {
        *sc = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        *m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

/* Unpacks one super-block into its 256 integer quants (0..15 for Q4_K, 0..31 for Q5_K),
 * element order of dequantize_block_q4_K / _q5_K (quantized.cu:943-1004):
 * element 64j+l <- low nibble of qs[32j+l] (sub-block 2j), 64j+32+l <- high nibble (2j+1);
 * Q5_K adds 16 when bit 2j (resp. 2j+1) of qh[l] is set. */
static inline void unpack_quants(int gguf_type, const uint8_t *blk, uint8_t *qv, int *sc, int *mn,
                                 float *dall, float *dmin) {
    *dall = h2f(blk);
    *dmin = h2f(blk + 2);
    const uint8_t *scales = blk + 4;
    for (int j = 0; j < 8; ++j) scale_min_k4(j, scales, &sc[j], &mn[j]);
    if (gguf_type == ORC_Q4K) {
        const uint8_t *qs = blk + 16;
        for (int j = 0; j < 4; ++j)
            for (int l = 0; l < 32; ++l) {
                qv[64 * j + l] = qs[32 * j + l] & 0xF;
                qv[64 * j + 32 + l] = qs[32 * j + l] >> 4;
            }
    } else {
        const uint8_t *qh = blk + 16;
        const uint8_t *qs = blk + 48;
        for (int j = 0; j < 4; ++j)
            for (int l = 0; l < 32; ++l) {
                qv[64 * j + l] = (uint8_t)((qs[32 * j + l] & 0xF) + (((qh[l] >> (2 * j)) & 1) << 4));
                qv[64 * j + 32 + l] =
                    (uint8_t)((qs[32 * j + l] >> 4) + (((qh[l] >> (2 * j + 1)) & 1) << 4));
            }
    }
}

/* dequantize_block_q4_K / _q5_K in f32 (quantized.cu:935-1004): d1 = dall*sc, m1 = dmin*m,
 * y = d1*q - m1.  The reference's compiled kernel contracts the last step into one FMA. */
static void dequant_k(int gguf_type, const uint8_t *blocks, int64_t nblocks, float *out, int fused) {
    const size_t bb = gguf_type == ORC_Q4K ? ORC_Q4K_BYTES : ORC_Q5K_BYTES;
#pragma omp parallel for schedule(static)
    for (int64_t b = 0; b < nblocks; ++b) {
        uint8_t qv[256];
        int sc[8], mn[8];
        float dall, dmin;
        unpack_quants(gguf_type, blocks + b * bb, qv, sc, mn, &dall, &dmin);
        float *y = out + b * 256;
        for (int e = 0; e < 256; ++e) {
            const int s = e / 32;
            const float d1 = dall * (float)sc[s];
            const float m1 = dmin * (float)mn[s];
            y[e] = fused ? fmaf(d1, (float)qv[e], -m1) : (d1 * (float)qv[e]) - m1;
        }
    }
}

void orc_dequant_q4k(const uint8_t *blocks, int64_t nblocks, float *out, int fused) {
    dequant_k(ORC_Q4K, blocks, nblocks, out, fused);
}
void orc_dequant_q5k(const uint8_t *blocks, int64_t nblocks, float *out, int fused) {
    dequant_k(ORC_Q5K, blocks, nblocks, out, fused);
}

/* ------------------------------------------------------------------------------------ */
/* Q8_1 activation quantisation                                                          */
/* ------------------------------------------------------------------------------------ */
/* Sum of 32 lane values by xor-butterfly 16,8,4,2,1 (warp_reduce_sum, gguf.cuh:29-35).
 * Every lane ends with the same value because f32 addition is commutative. */
static inline float butterfly32(const float *v) {
    float a[32], b[32];
    memcpy(a, v, sizeof(a));
    for (int mask = 16; mask > 0; mask >>= 1) {
        for (int l = 0; l < 32; ++l) b[l] = a[l] + a[l ^ mask];
        memcpy(a, b, sizeof(a));
    }
    return a[0];
}

/* quantize_q8_1 (gguf.cuh:1234-1261). */
void orc_quantize_q8_1(const float *x, int rows, int k, int kpad, uint8_t *out) {
    const int nb = kpad / 32;
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r) {
        for (int b = 0; b < nb; ++b) {
            float v[32];
            float amax = 0.0f;
            for (int l = 0; l < 32; ++l) {
                const int ix = b * 32 + l;
                v[l] = ix < k ? x[(size_t)r * k + ix] : 0.0f;
                amax = fmaxf(amax, fabsf(v[l]));
            }
            const float sum = butterfly32(v);
            const float d = amax / 127.0f;
            uint8_t *blk = out + ((size_t)r * nb + b) * ORC_Q81_BYTES;
            for (int l = 0; l < 32; ++l) {
                const int8_t q = amax == 0.0f ? 0 : (int8_t)roundf(v[l] / d);
                blk[4 + l] = (uint8_t)q;
            }
            const uint16_t hd = orc_float_to_half(d), hs = orc_float_to_half(sum);
            memcpy(blk, &hd, 2);
            memcpy(blk + 2, &hs, 2);
        }
    }
}

/* quantize_mmq_q8_1<DS4> (mmq_quantize.cu:11-107): 8 threads x 4 values per 32-block;
 * sum = (((x0+x1)+x2)+x3) per thread, then xor-butterfly over offsets 4,2,1. */
static inline void quant_mmq_block(const float *v, int8_t *q, uint16_t *d, uint16_t *s) {
    float amax = 0.0f;
    for (int l = 0; l < 32; ++l) amax = fmaxf(amax, fabsf(v[l]));
    float t[8], u[8];
    for (int i = 0; i < 8; ++i) t[i] = ((v[4 * i] + v[4 * i + 1]) + v[4 * i + 2]) + v[4 * i + 3];
    for (int off = 4; off > 0; off >>= 1) {
        for (int i = 0; i < 8; ++i) u[i] = t[i] + t[i ^ off];
        memcpy(t, u, sizeof(t));
    }
    if (amax == 0.0f) {
        /* d_inv = inf: 0*inf is NaN and the int8 conversion of NaN yields 0; d = 1/inf = 0. */
        for (int l = 0; l < 32; ++l) q[l] = 0;
        *d = orc_float_to_half(0.0f);
    } else {
        const float d_inv = 127.0f / amax;
        for (int l = 0; l < 32; ++l) q[l] = (int8_t)roundf(v[l] * d_inv);
        *d = orc_float_to_half(1.0f / d_inv);
    }
    *s = orc_float_to_half(t[0]);
}

void orc_quantize_q8_1_mmq(const float *x, const int32_t *src_rows, int rows, int k, int kpad,
                           int8_t *q, uint16_t *d, uint16_t *s) {
    const int nb = kpad / 32;
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r) {
        const int64_t src = src_rows ? src_rows[r] : r;
        for (int b = 0; b < nb; ++b) {
            float v[32];
            for (int l = 0; l < 32; ++l) {
                const int ix = b * 32 + l;
                v[l] = ix < k ? x[(size_t)src * k + ix] : 0.0f;
            }
            quant_mmq_block(v, q + (size_t)r * kpad + b * 32, d + (size_t)r * nb + b,
                            s + (size_t)r * nb + b);
        }
    }
}

/* ------------------------------------------------------------------------------------ */
/* Row dot products                                                                      */
/* ------------------------------------------------------------------------------------ */
/* Integer part of a super-block x Q8_1 dot: per 32-element sub-block the quant dot and the
 * activation sum (the dp4a-with-ones term of vec_dot_q4_K_q8_1_impl_vmmq, gguf.cuh:727-750). */
HOT static void kq_subdots(int gguf_type, const uint8_t *blk, const int8_t *a, int *dot) {
    if (gguf_type == ORC_Q4K) {
        const uint8_t *qs = blk + 16;
        for (int j = 0; j < 4; ++j) {
            int lo = 0, hi = 0;
            for (int l = 0; l < 32; ++l) {
                lo += (qs[32 * j + l] & 0xF) * a[64 * j + l];
                hi += (qs[32 * j + l] >> 4) * a[64 * j + 32 + l];
            }
            dot[2 * j] = lo;
            dot[2 * j + 1] = hi;
        }
    } else {
        const uint8_t *qh = blk + 16;
        const uint8_t *qs = blk + 48;
        for (int j = 0; j < 4; ++j) {
            int lo = 0, hi = 0;
            for (int l = 0; l < 32; ++l) {
                const int ql = (qs[32 * j + l] & 0xF) | (((qh[l] >> (2 * j)) & 1) << 4);
                const int qq = (qs[32 * j + l] >> 4) | (((qh[l] >> (2 * j + 1)) & 1) << 4);
                lo += ql * a[64 * j + l];
                hi += qq * a[64 * j + 32 + l];
            }
            dot[2 * j] = lo;
            dot[2 * j + 1] = hi;
        }
    }
}

/* MMVQ combine (gguf.cuh:727-750 / 783-813): per super-block
 * dall * sum_i d8_i*(dot_i*sc_i) - dmin * sum_i d8_i*(sumq_i*m_i). */
static float dot_kq_q81(int gguf_type, const uint8_t *wrow, const uint8_t *q81row, int nsb) {
    const size_t bb = gguf_type == ORC_Q4K ? ORC_Q4K_BYTES : ORC_Q5K_BYTES;
    float acc = 0.0f;
    for (int b = 0; b < nsb; ++b) {
        const uint8_t *blk = wrow + b * bb;
        int8_t a[256];
        float d8[8];
        int sumq[8];
        for (int s = 0; s < 8; ++s) {
            const uint8_t *q8 = q81row + (size_t)(b * 8 + s) * ORC_Q81_BYTES;
            d8[s] = h2f(q8);
            int t = 0;
            for (int l = 0; l < 32; ++l) {
                a[32 * s + l] = (int8_t)q8[4 + l];
                t += (int8_t)q8[4 + l];
            }
            sumq[s] = t;
        }
        int dot[8];
        kq_subdots(gguf_type, blk, a, dot);
        int sc[8], mn[8];
        for (int j = 0; j < 8; ++j) scale_min_k4(j, blk + 4, &sc[j], &mn[j]);
        float sumf_d = 0.0f, sumf_m = 0.0f;
        for (int s = 0; s < 8; ++s) {
            sumf_d += d8[s] * (float)(dot[s] * sc[s]);
            sumf_m += d8[s] * (float)(sumq[s] * mn[s]);
        }
        acc += h2f(blk) * sumf_d - h2f(blk + 2) * sumf_m;
    }
    return acc;
}

float orc_dot_q4k_q81(const uint8_t *wrow, const uint8_t *q81row, int nsb) {
    return dot_kq_q81(ORC_Q4K, wrow, q81row, nsb);
}
float orc_dot_q5k_q81(const uint8_t *wrow, const uint8_t *q81row, int nsb) {
    return dot_kq_q81(ORC_Q5K, wrow, q81row, nsb);
}

/* MMQ combine: the tile loader stores dmA = half2(dall,-dmin) * half2(sc, m) rounded to half
 * (mmq_gguf.cuh:2115-2121, 2283-2289); vec_dot_q8_1_q8_1_mma adds dmA.x*dsB.x*C + dmA.y*dsB.y
 * per 32-block in K order (mmq_gguf.cuh:1210-1214). */
float orc_dot_kq_mmq(int gguf_type, const uint8_t *wrow, const int8_t *q, const uint16_t *d,
                     const uint16_t *s, int nsb) {
    const size_t bb = gguf_type == ORC_Q4K ? ORC_Q4K_BYTES : ORC_Q5K_BYTES;
    float sum = 0.0f;
    for (int b = 0; b < nsb; ++b) {
        const uint8_t *blk = wrow + b * bb;
        int dot[8];
        kq_subdots(gguf_type, blk, q + b * 256, dot);
        const float dall = h2f(blk), ndmin = -h2f(blk + 2);
        for (int j = 0; j < 8; ++j) {
            int sc, mn;
            scale_min_k4(j, blk + 4, &sc, &mn);
            const float dmx = orc_half_to_float(orc_float_to_half(dall * (float)sc));
            const float dmy = orc_half_to_float(orc_float_to_half(ndmin * (float)mn));
            const float dsx = orc_half_to_float(d[b * 8 + j]);
            const float dsy = orc_half_to_float(s[b * 8 + j]);
            sum = fmaf(dmx * dsx, (float)dot[j], sum);
            sum = fmaf(dmy, dsy, sum);
        }
    }
    return sum;
}

/* ------------------------------------------------------------------------------------ */
/* Routing                                                                               */
/* ------------------------------------------------------------------------------------ */
/* Canonical router dot: K is cut into 8 contiguous slices; in slice s, lane l (0..31) accumulates
 * the float4 groups l, l+32, ... of that slice with fmaf (components in order); the 32 lane
 * partials are summed by xor-butterfly and the 8 slice sums by ((s0+s1)+(s2+s3))+((s4+s5)+(s6+s7)).
 * The CUDA kernels compute exactly this order, so the logits are bit-identical. */
HOT static float router_dot(const float *x, const float *w, int K) {
    const int slice = K / 8, groups = slice / 4;
    float ss[8];
    for (int sl = 0; sl < 8; ++sl) {
        float lane[32];
        const float *xs = x + sl * slice, *ws = w + sl * slice;
        for (int l = 0; l < 32; ++l) {
            float acc = 0.0f;
            for (int g = l; g < groups; g += 32) {
                const int base = 4 * g;
                acc = fmaf(ws[base + 0], xs[base + 0], acc);
                acc = fmaf(ws[base + 1], xs[base + 1], acc);
                acc = fmaf(ws[base + 2], xs[base + 2], acc);
                acc = fmaf(ws[base + 3], xs[base + 3], acc);
            }
            lane[l] = acc;
        }
        ss[sl] = butterfly32(lane);
    }
    return ((ss[0] + ss[1]) + (ss[2] + ss[3])) + ((ss[4] + ss[5]) + (ss[6] + ss[7]));
}

void orc_router_logits(const float *x, const float *wr, int T, int E, int K, float *logits) {
#pragma omp parallel for collapse(2) schedule(static)
    for (int t = 0; t < T; ++t)
        for (int e = 0; e < E; ++e)
            logits[(size_t)t * E + e] = router_dot(x + (size_t)t * K, wr + (size_t)e * K, K);
}

/* Tree sum of the selected weights: strides topk/2, topk/4, ..., 1 (moe_gguf.cu:63-68 for 8). */
static float tree_sum(const float *v, int n) {
    float a[64];
    memcpy(a, v, sizeof(float) * n);
    if (n & (n - 1)) { /* not a power of two: sequential */
        float s = 0.0f;
        for (int i = 0; i < n; ++i) s += a[i];
        return s;
    }
    for (int st = n / 2; st > 0; st /= 2)
        for (int i = 0; i < st; ++i) a[i] = a[i] + a[i + st];
    return a[0];
}

static void route_one(const float *logits, const float *bias, int E, int topk, uint32_t *ids,
                      float *w) {
    float s[1024], sel[1024];
    for (int e = 0; e < E; ++e) {
        s[e] = 1.0f / (1.0f + expf(-logits[e]));
        sel[e] = s[e] + bias[e];
        if (sel[e] == 0.0f) sel[e] = 0.0f; /* -0 and +0 rank as equal */
    }
    /* rank_e = #{j: sel_j > sel_e} + #{j < e: sel_j == sel_e} (stable descending order). */
    for (int e = 0; e < E; ++e) {
        int rank = 0;
        for (int j = 0; j < E && rank < topk; ++j)
            rank += (sel[j] > sel[e]) || (sel[j] == sel[e] && j < e);
        if (rank < topk) ids[rank] = (uint32_t)e;
    }
    float sw[64] = {0};
    for (int k = 0; k < topk; ++k) sw[k] = s[ids[k]];
    const float denom = tree_sum(sw, topk);
    for (int k = 0; k < topk; ++k) w[k] = sw[k] / denom;
}

void orc_route_topk(const float *logits, const float *bias, int T, int E, int topk,
                    uint32_t *topk_ids, float *topk_w) {
#pragma omp parallel for schedule(static)
    for (int t = 0; t < T; ++t)
        route_one(logits + (size_t)t * E, bias, E, topk, topk_ids + (size_t)t * topk,
                  topk_w + (size_t)t * topk);
}

void orc_decode_topk(const float *logits, const float *bias, uint32_t *topk_ids, float *topk_w,
                     uint32_t *expert_ids, uint32_t *route_ids) {
    route_one(logits, bias, 256, 8, topk_ids, topk_w);
    /* insertion sort of (expert, slot) by expert id (moe_gguf.cu:77-90) */
    uint32_t e[8], r[8];
    for (int i = 0; i < 8; ++i) {
        e[i] = topk_ids[i];
        r[i] = (uint32_t)i;
    }
    for (int i = 1; i < 8; ++i) {
        const uint32_t key = e[i], rt = r[i];
        int j = i - 1;
        while (j >= 0 && e[j] > key) {
            e[j + 1] = e[j];
            r[j + 1] = r[j];
            --j;
        }
        e[j + 1] = key;
        r[j + 1] = rt;
    }
    memcpy(expert_ids, e, sizeof(e));
    memcpy(route_ids, r, sizeof(r));
}

void orc_sort_routes(const uint32_t *expert_ids, int n, uint32_t *sorted_experts,
                     uint32_t *sorted_routes) {
    uint32_t maxe = 0;
    for (int i = 0; i < n; ++i)
        if (expert_ids[i] > maxe) maxe = expert_ids[i];
    int *off = (int *)calloc((size_t)maxe + 2, sizeof(int));
    for (int i = 0; i < n; ++i) off[expert_ids[i] + 1]++;
    for (uint32_t e = 0; e <= maxe; ++e) off[e + 1] += off[e];
    for (int i = 0; i < n; ++i) {
        const int p = off[expert_ids[i]]++;
        sorted_experts[p] = expert_ids[i];
        sorted_routes[p] = (uint32_t)i;
    }
    free(off);
}

/* ------------------------------------------------------------------------------------ */
/* Expert GEMMs                                                                          */
/* ------------------------------------------------------------------------------------ */
void orc_moe_gemm_gguf(const float *input, const uint8_t *weights, const int32_t *sorted_token_ids,
                       const int32_t *expert_ids, const float *topk_weights, float *output,
                       int num_experts, int topk, int size_m, int size_n, int size_k,
                       int gguf_type) {
    const int kpad = pad_to(size_k, 512);
    const int m = topk_weights ? size_m : size_m / topk;
    const int nb = kpad / 32;
    uint8_t *q = (uint8_t *)malloc((size_t)m * nb * ORC_Q81_BYTES);
    orc_quantize_q8_1(input, m, size_k, kpad, q);
    const size_t rb = orc_row_bytes(gguf_type, size_k);
    const size_t es = rb * (size_t)size_n;
#pragma omp parallel for collapse(2) schedule(static)
    for (int i = 0; i < size_m; ++i)
        for (int row = 0; row < size_n; ++row) {
            const int token_id = sorted_token_ids[i];
            const int expert = expert_ids[i];
            if (expert < 0 || expert >= num_experts) continue;
            const float scale = topk_weights ? topk_weights[token_id] : 1.0f;
            const int in_row = topk_weights ? token_id : token_id / topk;
            const float v = dot_kq_q81(gguf_type, weights + (size_t)expert * es + row * rb,
                                       q + (size_t)in_row * nb * ORC_Q81_BYTES, size_k / 256);
            output[(size_t)token_id * size_n + row] = v * scale;
        }
    free(q);
}

void orc_moe_gemm_mmq(const float *input, const uint8_t *weights, const int32_t *sorted_token_ids,
                      const int32_t *expert_ids, const float *topk_weights, float *output,
                      int num_experts, int topk, int size_m, int size_n, int size_k,
                      int gguf_type) {
    if (gguf_type != ORC_Q4K && gguf_type != ORC_Q5K) return; /* mmq_moe.cu:84-86 */
    const int kpad = pad_to(size_k, 512);
    const int nb = kpad / 32;
    const int id_div = topk_weights ? 1 : topk;
    int32_t *src = (int32_t *)malloc(sizeof(int32_t) * size_m);
    for (int i = 0; i < size_m; ++i) src[i] = sorted_token_ids[i] / id_div;
    int8_t *q = (int8_t *)malloc((size_t)size_m * kpad);
    uint16_t *d = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)size_m * nb);
    uint16_t *s = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)size_m * nb);
    orc_quantize_q8_1_mmq(input, src, size_m, size_k, kpad, q, d, s);
    const size_t rb = orc_row_bytes(gguf_type, size_k);
    const size_t es = rb * (size_t)size_n;
#pragma omp parallel for collapse(2) schedule(static)
    for (int i = 0; i < size_m; ++i)
        for (int row = 0; row < size_n; ++row) {
            const int expert = expert_ids[i];
            if (expert < 0 || expert >= num_experts) continue;
            const int token_id = sorted_token_ids[i];
            float v = orc_dot_kq_mmq(gguf_type, weights + (size_t)expert * es + row * rb,
                                     q + (size_t)i * kpad, d + (size_t)i * nb, s + (size_t)i * nb,
                                     size_k / 256);
            output[(size_t)token_id * size_n + row] = v;
        }
    if (topk_weights) { /* scale_moe_rows (mmq_moe.cu:58-67) */
#pragma omp parallel for schedule(static)
        for (int r = 0; r < size_m; ++r)
            for (int n = 0; n < size_n; ++n) output[(size_t)r * size_n + n] *= topk_weights[r];
    }
    free(src);
    free(q);
    free(d);
    free(s);
}

static inline float silu_mul(float g, float u) { return u * (g / (1.0f + expf(-g))); }

void orc_moe_decode_silu(const float *input, const uint8_t *gate_w, const uint8_t *up_w,
                         const uint8_t *down_w, const int32_t *sorted_token_ids,
                         const int32_t *expert_ids, const float *topk_weights, float *output,
                         int num_experts, int topk, int hidden, int inter, int gate_up_type,
                         int down_type) {
    if (topk != 8) return; /* moe_gguf.cu:457-459 */
    const int hpad = pad_to(hidden, 512), ipad = pad_to(inter, 512);
    uint8_t *xq = (uint8_t *)malloc((size_t)(hpad / 32) * ORC_Q81_BYTES);
    orc_quantize_q8_1(input, 1, hidden, hpad, xq);
    float *g = (float *)calloc((size_t)topk * inter, sizeof(float));
    float *u = (float *)calloc((size_t)topk * inter, sizeof(float));
    const size_t grb = orc_row_bytes(gate_up_type, hidden);
    const size_t drb = orc_row_bytes(down_type, inter);
#pragma omp parallel for collapse(2) schedule(static)
    for (int i = 0; i < topk; ++i)
        for (int n = 0; n < inter; ++n) {
            const int slot = sorted_token_ids[i], e = expert_ids[i];
            if (e < 0 || e >= num_experts) continue;
            const size_t off = ((size_t)e * inter + n) * grb;
            g[(size_t)slot * inter + n] = dot_kq_q81(gate_up_type, gate_w + off, xq, hidden / 256);
            u[(size_t)slot * inter + n] = dot_kq_q81(gate_up_type, up_w + off, xq, hidden / 256);
        }
    float *a = (float *)malloc(sizeof(float) * (size_t)topk * inter);
    for (size_t i = 0; i < (size_t)topk * inter; ++i) a[i] = silu_mul(g[i], u[i]);
    uint8_t *aq = (uint8_t *)malloc((size_t)topk * (ipad / 32) * ORC_Q81_BYTES);
    orc_quantize_q8_1(a, topk, inter, ipad, aq);
#pragma omp parallel for schedule(static)
    for (int r = 0; r < hidden; ++r) {
        float v[8] = {0};
        for (int i = 0; i < topk; ++i) {
            const int slot = sorted_token_ids[i], e = expert_ids[i];
            if (e < 0 || e >= num_experts) continue;
            const float dv = dot_kq_q81(down_type, down_w + ((size_t)e * hidden + r) * drb,
                                        aq + (size_t)slot * (ipad / 32) * ORC_Q81_BYTES,
                                        inter / 256);
            v[slot] = dv * topk_weights[slot];
        }
        /* fixed 8-way tree (moe_gguf.cu:328-342) */
        output[r] = ((v[0] + v[4]) + (v[2] + v[6])) + ((v[1] + v[5]) + (v[3] + v[7]));
    }
    free(xq);
    free(g);
    free(u);
    free(a);
    free(aq);
}

/* ------------------------------------------------------------------------------------ */
/* The MoE block                                                                         */
/* ------------------------------------------------------------------------------------ */
void orc_moe_block(const OrcMoeWeights *w, const float *x, const float *residual, int T,
                   int mmq_min_tokens, float *y, uint32_t *topk_ids, float *topk_w) {
    const int E = w->num_experts, K = w->topk, H = w->hidden, I = w->inter;
    float *logits = (float *)malloc(sizeof(float) * (size_t)T * E);
    orc_router_logits(x, w->router, T, E, H, logits);
    uint32_t *ids = (uint32_t *)malloc(sizeof(uint32_t) * (size_t)T * K);
    float *tw = (float *)malloc(sizeof(float) * (size_t)T * K);
    if (T == 1 && E == 256 && K == 8) {
        uint32_t eids[8], rids[8];
        orc_decode_topk(logits, w->bias, ids, tw, eids, rids);
        int32_t se[8], sr[8];
        for (int i = 0; i < 8; ++i) {
            se[i] = (int32_t)eids[i];
            sr[i] = (int32_t)rids[i];
        }
        orc_moe_decode_silu(x, w->gate, w->up, w->down, sr, se, tw, y, E, K, H, I,
                            w->gate_up_type, w->down_type);
    } else {
        orc_route_topk(logits, w->bias, T, E, K, ids, tw);
        const int M = T * K;
        uint32_t *se = (uint32_t *)malloc(sizeof(uint32_t) * M);
        uint32_t *sr = (uint32_t *)malloc(sizeof(uint32_t) * M);
        orc_sort_routes(ids, M, se, sr);
        float *g = (float *)malloc(sizeof(float) * (size_t)M * I);
        float *u = (float *)malloc(sizeof(float) * (size_t)M * I);
        float *dn = (float *)malloc(sizeof(float) * (size_t)M * H);
        const int mmq = T >= mmq_min_tokens && (w->gate_up_type == ORC_Q4K || w->gate_up_type == ORC_Q5K);
        void (*gemm)(const float *, const uint8_t *, const int32_t *, const int32_t *,
                     const float *, float *, int, int, int, int, int, int) =
            mmq ? orc_moe_gemm_mmq : orc_moe_gemm_gguf;
        gemm(x, w->gate, (const int32_t *)sr, (const int32_t *)se, NULL, g, E, K, M, I, H,
             w->gate_up_type);
        gemm(x, w->up, (const int32_t *)sr, (const int32_t *)se, NULL, u, E, K, M, I, H,
             w->gate_up_type);
        for (size_t i = 0; i < (size_t)M * I; ++i) g[i] = silu_mul(g[i], u[i]);
        const int mmq_down = T >= mmq_min_tokens && (w->down_type == ORC_Q4K || w->down_type == ORC_Q5K);
        (mmq_down ? orc_moe_gemm_mmq : orc_moe_gemm_gguf)(g, w->down, (const int32_t *)sr,
                                                          (const int32_t *)se, tw, dn, E, K, M, H,
                                                          I, w->down_type);
        for (int t = 0; t < T; ++t)
            for (int h = 0; h < H; ++h) {
                float s = 0.0f;
                for (int k = 0; k < K; ++k) s += dn[((size_t)t * K + k) * H + h];
                y[(size_t)t * H + h] = s;
            }
        free(se);
        free(sr);
        free(g);
        free(u);
        free(dn);
    }
    if (residual)
        for (size_t i = 0; i < (size_t)T * H; ++i) y[i] = y[i] + residual[i];
    if (topk_ids) memcpy(topk_ids, ids, sizeof(uint32_t) * (size_t)T * K);
    if (topk_w) memcpy(topk_w, tw, sizeof(float) * (size_t)T * K);
    free(logits);
    free(ids);
    free(tw);
}
