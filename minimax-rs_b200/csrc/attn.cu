// Single-token attention half of a MiniMax-M2.7 layer on B200 (sm_100a).
//
// Reference path (minimax-rs, src/model.rs:79-162, T = 1): q8_0_decode_rmsnorm_f16
// (candle-nn fused_qkv.rs:162-280 -> mmvq_gguf.cu:814-885), partial_rope_f16
// (mmvq_gguf.cu:1038-1066), KV-cache append, gqa_decode_f16_128 (fused_attention.rs:21-42 ->
// decode_attention.cu:311-918) and the Q8_0 output projection (QMatMul: quantize_q8_1 +
// mmvq, mmvq_gguf.cu:1137-1200).
//
// All of it is memory-bound (Q8_0 weights 46.8 MB and the f16 KV cache per token), so the kernels
// are dp4a / packed-f32 CUDA-core kernels that keep every byte moving once:
//   * matvec: each CTA quantises the activation into shared memory, a warp owns a row and its
//     lanes stride over the 34-byte Q8_0 blocks, read as aligned 32-bit words and realigned with
//     funnel shifts (k % 64 == 0 keeps the last word of every block inside its row);
//   * attention: CTA = (key split, KV head); a lane owns a key for Q.K (its 256-byte K row against
//     the 6 query heads in shared memory), online softmax per warp, then a lane owns 4 dims for
//     P.V (coalesced V rows); warps merge in shared memory; a combine kernel merges the splits.
#include <cuda_fp16.h>

#include <algorithm>
#include <cfloat>
#include <mutex>

#include "../../include/minimax_attn.h"
#include "common.cuh"
#include "workspace.cuh"

namespace mmrs {

constexpr int kAttnHeadDim = 128;
constexpr int kAttnGroup = 6;            // query heads per KV head
constexpr int kAttnPartial = kAttnHeadDim + 2;  // (max, sum, 128 unnormalised values)
constexpr int kAttnMaxSplits = 128;
constexpr int kMvThreads = 256;          // matvec CTA: 8 warps, one row per warp at a time
constexpr int kMvMaxK = 8192;

// ------------------------------------------------------------------------------------------
// Q8_1 of one 32-element block (quantize_q8_1, mmvq_gguf.cu:1137-1169): lane = element;
// d = amax / 127, q = roundf(x / d); the block's half d (for the dot) and half sum.
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ int8_t q81_lane(float x, float &d_out, float &sum_out) {
    float amax = fabsf(x), sum = x;
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) {
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, m));
        sum += __shfl_xor_sync(0xffffffffu, sum, m);
    }
    const float d = __fdiv_rn(amax, 127.0f);
    d_out = d;
    sum_out = sum;
    return amax == 0.0f ? (int8_t)0 : (int8_t)roundf(__fdiv_rn(x, d));
}

// Activation in shared memory: int8 quants [k] and the per-block half d as float [k / 32].
struct MvAct {
    int8_t *q;
    float *d;
};

// Quantise x (f32 or f16) into shared memory (all threads of the CTA); optionally also store the
// Q8_1 blocks in the reference's 36-byte layout (vy, zero-padded to kpad).
template <typename T>
__device__ void mv_quantize(const T *__restrict__ x, int k, MvAct a, uint8_t *vy, int kpad) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    for (int b = warp; b < kpad / 32; b += nw) {
        const int i = b * 32 + lane;
        const float v = i < k ? (float)x[i] : 0.0f;
        float d, sum;
        const int8_t q = q81_lane(v, d, sum);
        if (b < k / 32) {  // k % 32 == 0: blocks past k are only padding of vy
            a.q[i] = q;
            if (lane == 0) a.d[b] = __half2float(__float2half_rn(d));
        }
        if (vy) {
            uint8_t *blk = vy + (size_t)b * 36;
            blk[4 + lane] = (uint8_t)q;
            if (lane == 0) {
                const __half hd = __float2half_rn(d), hs = __float2half_rn(sum);
                *reinterpret_cast<__half *>(blk) = hd;
                *reinterpret_cast<__half *>(blk + 2) = hs;
            }
        }
    }
}

// Dot of Q8_0 row `row` (nb blocks of 34 bytes, nb even) with the shared-memory activation; the
// lanes of a warp stride over the blocks, the result is returned on every lane.
__device__ __forceinline__ float mv_row_dot(const uint8_t *__restrict__ row, int nb, MvAct a, int lane) {
    float acc = 0.0f;
    for (int b = lane; b < nb; b += 32) {
        // the block's 34 bytes from 9 aligned words: even b starts on a word, odd b two bytes in
        const uint32_t *w = reinterpret_cast<const uint32_t *>(row + ((34 * b) & ~3));
        uint32_t W[9];
#pragma unroll
        for (int i = 0; i < 9; ++i) W[i] = __ldg(w + i);
        const bool odd = b & 1;
        const uint32_t sh = odd ? 32u : 16u;
        const float dw = __half2float(__ushort_as_half((unsigned short)((odd ? W[0] >> 16 : W[0]) & 0xFFFFu)));
        const int4 *xq = reinterpret_cast<const int4 *>(a.q + 32 * b);
        const int4 x0 = xq[0], x1 = xq[1];
        const int xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
        int s0 = 0, s1 = 0;
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
            s0 = __dp4a((int)__funnelshift_rc(W[i], W[i + 1], sh), xv[i], s0);
            s1 = __dp4a((int)__funnelshift_rc(W[i + 1], W[i + 2], sh), xv[i + 1], s1);
        }
        // vec_dot_q8_0_q8_1_impl (mmvq_gguf.cu:282-290): sumi * d_w * d_x
        acc += __fmul_rn(__fmul_rn((float)(s0 + s1), dw), a.d[b]);
    }
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, m);
    return acc;
}

// One or more Q8_0 matrices sharing one activation: rows [0, n0) of w0, then n1 rows of w1, then
// n2 rows of w2, into dst [n0 + n1 + n2] (+ residual when given).  The activation is x (f32 or
// f16, quantised per CTA) or, with x == nullptr, ready Q8_1 blocks in vy_in.
struct MvParams {
    const uint8_t *w[3];
    int n[3];
    int k;
    const void *x;
    const uint8_t *vy_in;
    uint8_t *vy_out;  // CTA 0 stores the Q8_1 blocks here (kpad / 32 blocks) when not null
    int kpad;
    const float *residual;
    float *dst;
};

template <typename T>
__global__ void __launch_bounds__(kMvThreads) q8_0_matvec_kernel(const MvParams p) {
    extern __shared__ __align__(16) uint8_t mv_smem[];
    MvAct a{reinterpret_cast<int8_t *>(mv_smem), reinterpret_cast<float *>(mv_smem + p.kpad)};
    const int nb = p.k / 32;
    if (p.x) {
        mv_quantize<T>(static_cast<const T *>(p.x), p.k, a, blockIdx.x == 0 ? p.vy_out : nullptr, p.kpad);
    } else {
        for (int b = threadIdx.x; b < nb; b += blockDim.x) {
            const uint8_t *blk = p.vy_in + (size_t)b * 36;
            a.d[b] = __half2float(*reinterpret_cast<const __half *>(blk));
            // 36-byte blocks keep 4-byte alignment only: copy the quants as words
            const int *s32 = reinterpret_cast<const int *>(blk + 4);
            int *d32 = reinterpret_cast<int *>(a.q + 32 * b);
#pragma unroll
            for (int i = 0; i < 8; ++i) d32[i] = s32[i];
        }
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int total = p.n[0] + p.n[1] + p.n[2];
    const size_t row_bytes = (size_t)nb * 34;
    for (int r = blockIdx.x * (kMvThreads / 32) + warp; r < total; r += gridDim.x * (kMvThreads / 32)) {
        // matrix by comparison (indexing the parameter arrays would copy them to local memory)
        const bool m0 = r < p.n[0], m1 = !m0 && r < p.n[0] + p.n[1];
        const uint8_t *wm = m0 ? p.w[0] : (m1 ? p.w[1] : p.w[2]);
        const int rl = m0 ? r : (m1 ? r - p.n[0] : r - p.n[0] - p.n[1]);
        const float v = mv_row_dot(wm + (size_t)rl * row_bytes, nb, a, lane);
        if (lane == 0) p.dst[r] = p.residual ? v + p.residual[r] : v;
    }
}

static size_t mv_smem_bytes(int kpad) { return (size_t)kpad + (size_t)(kpad / 32) * sizeof(float); }

template <typename T>
static int mv_launch(const MvParams &p, cudaStream_t s) {
    const int total = p.n[0] + p.n[1] + p.n[2];
    if (p.k <= 0 || p.k % 64 || p.k > kMvMaxK || p.kpad < p.k || p.kpad % 32 || total <= 0) return MMRS_ERR_ARG;
    for (int m = 0; m < 3; ++m)
        if (p.n[m] > 0 && (!p.w[m] || ((uintptr_t)p.w[m] & 3u))) return MMRS_ERR_ARG;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int rows_per_cta = kMvThreads / 32;
    const int blocks = std::min((total + rows_per_cta - 1) / rows_per_cta, sms * 8);
    q8_0_matvec_kernel<T><<<blocks, kMvThreads, mv_smem_bytes(p.kpad), s>>>(p);
    return cudaGetLastError() == cudaSuccess ? MMRS_OK : MMRS_ERR_LAUNCH;
}

// ------------------------------------------------------------------------------------------
// Q / K RMSNorm to f16 (qkv_rmsnorm_f16_cuda1, mmvq_gguf.cu:838-885): CTA 0 = q, 1 = k, 2 = v
// (copy); sum of squares in a fixed order (thread-strided partials, warp tree, block tree).
// ------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) qkv_rmsnorm_f16_kernel(const float *__restrict__ src,
                                                               const float *__restrict__ qa,
                                                               const float *__restrict__ ka, __half *__restrict__ dst,
                                                               int q_rows, int k_rows, int v_rows, float eps) {
    __shared__ float ws[32];
    const int proj = blockIdx.x, tid = threadIdx.x;
    const int n = proj == 0 ? q_rows : (proj == 1 ? k_rows : v_rows);
    const int off = proj == 0 ? 0 : (proj == 1 ? q_rows : q_rows + k_rows);
    if (proj == 2) {
        for (int i = tid; i < n; i += blockDim.x) dst[off + i] = __float2half_rn(src[off + i]);
        return;
    }
    float ss = 0.0f;
    for (int i = tid; i < n; i += blockDim.x) ss = fmaf(src[off + i], src[off + i], ss);
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, m);
    if ((tid & 31) == 0) ws[tid >> 5] = ss;
    __syncthreads();
    float t = (tid & 31) < (int)(blockDim.x >> 5) ? ws[tid & 31] : 0.0f;
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) t += __shfl_xor_sync(0xffffffffu, t, m);
    const float scale = rsqrtf(__fdiv_rn(t, (float)n) + eps);
    const float *alpha = proj == 0 ? qa : ka;
    for (int i = tid; i < n; i += blockDim.x) dst[off + i] = __float2half_rn(__fmul_rn(__fmul_rn(scale, src[off + i]), alpha[i]));
}

// ------------------------------------------------------------------------------------------
// Partial rotary embedding (partial_rope_f16_cuda1, mmvq_gguf.cu:1038-1066), thread per output
// element of [Q rows | K rows]: columns >= rope_dim of a head are copied; the first half of the
// rotated columns is fma(x, c, -rn(x' * s)), the second fma(x', s, rn(x * c)) in half, c / s the
// f32 table entries rounded to half (the arithmetic of the reference kernel as compiled, written
// with explicit fma so that it does not depend on contraction).  K (and V, when given) go to
// k_out / v_out at (local / head_dim) * kv_stride + local % head_dim: kv_stride = head_dim for a
// contiguous output, the cache's per-head stride to append one position to a KV cache.
// ------------------------------------------------------------------------------------------
struct RopeParams {
    const __half *q, *k, *v;
    const float *cos, *sin;
    __half *q_out, *k_out, *v_out;
    int q_rows, k_rows, head_dim, rope_dim, position;
    long kv_stride;
};

__global__ void __launch_bounds__(256) partial_rope_kernel(const RopeParams p) {
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= p.q_rows + 2 * p.k_rows) return;
    if (idx >= p.q_rows + p.k_rows) {  // V copy (cache append only)
        if (!p.v) return;
        const int local = idx - p.q_rows - p.k_rows;
        p.v_out[(long)(local / p.head_dim) * p.kv_stride + local % p.head_dim] = p.v[local];
        return;
    }
    const bool is_q = idx < p.q_rows;
    const int local = is_q ? idx : idx - p.q_rows;
    const __half *src = is_q ? p.q : p.k;
    __half *dst = is_q ? p.q_out + local : p.k_out + (long)(local / p.head_dim) * p.kv_stride + local % p.head_dim;
    const int col = local % p.head_dim;
    if (col >= p.rope_dim) {
        *dst = src[local];
        return;
    }
    const int half_rope = p.rope_dim / 2;
    const bool first = col < half_rope;
    const int pair = first ? local + half_rope : local - half_rope;
    const int freq = first ? col : col - half_rope;
    const __half c = __float2half_rn(p.cos[p.position * half_rope + freq]);
    const __half sn = __float2half_rn(p.sin[p.position * half_rope + freq]);
    *dst = first ? __hfma(src[local], c, __hneg(__hmul_rn(src[pair], sn)))
                 : __hfma(src[pair], sn, __hmul_rn(src[local], c));
}

// ------------------------------------------------------------------------------------------
// Split-K GQA decode.  CTA = (split, KV head g), 4 warps; the split's keys [k0, k1) are walked
// in 32-key chunks, chunk c by warp c % 4.  Q.K: lane = key, its K row (16 x 16 B) against the
// 6 query heads held in shared memory (packed f32 FMAs); online softmax per warp and head; P.V:
// lane = 4 dims, each key's probability broadcast by shuffle, V rows read coalesced.  The warps'
// (max, sum, values) merge in shared memory into the split's partial per query head.
// ------------------------------------------------------------------------------------------
struct GqaParams {
    const __half *q, *k, *v;
    float *partials;
    int seq_len, q_head_stride, num_splits, query_heads;
    long k_head_stride, v_head_stride;
    float scale;
};

__device__ __forceinline__ float2 h2f2(uint32_t h) {
    return __half22float2(*reinterpret_cast<const __half2 *>(&h));
}

__global__ void __launch_bounds__(128) gqa_decode_kernel(const GqaParams p) {
    __shared__ __align__(16) float qs[kAttnGroup][kAttnHeadDim];
    __shared__ float wm[4][kAttnGroup], wl[4][kAttnGroup];
    __shared__ __align__(16) float wacc[4][kAttnGroup][kAttnHeadDim];
    const int split = blockIdx.x, g = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int k0 = (int)((long)p.seq_len * split / p.num_splits);
    const int k1 = (int)((long)p.seq_len * (split + 1) / p.num_splits);
    for (int i = tid; i < kAttnGroup * kAttnHeadDim; i += blockDim.x) {
        const int h = i / kAttnHeadDim, d = i % kAttnHeadDim;
        qs[h][d] = __half2float(p.q[(long)(g * kAttnGroup + h) * p.q_head_stride + d]);
    }
    __syncthreads();
    const __half *kh = p.k + (long)g * p.k_head_stride, *vh = p.v + (long)g * p.v_head_stride;
    float m[kAttnGroup], l[kAttnGroup], acc[kAttnGroup][4];
#pragma unroll
    for (int h = 0; h < kAttnGroup; ++h) {
        m[h] = -INFINITY;
        l[h] = 0.0f;
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[h][j] = 0.0f;
    }
    const int nchunks = (k1 - k0 + 31) / 32;
    for (int c = warp; c < nchunks; c += 4) {
        const int base = k0 + 32 * c, nvalid = min(32, k1 - base);
        const bool valid = lane < nvalid;
        float sc[kAttnGroup];
        {
            float2 s2[kAttnGroup];
#pragma unroll
            for (int h = 0; h < kAttnGroup; ++h) s2[h] = make_float2(0.0f, 0.0f);
            if (valid) {
                // the lane's whole K row in flight at once (16 x 16 B)
                const uint4 *kr = reinterpret_cast<const uint4 *>(kh + (long)(base + lane) * kAttnHeadDim);
                uint4 krow[kAttnHeadDim / 8];
#pragma unroll
                for (int i = 0; i < kAttnHeadDim / 8; ++i) krow[i] = __ldg(kr + i);
#pragma unroll
                for (int i = 0; i < kAttnHeadDim / 8; ++i) {
                    const uint4 kv = krow[i];
                    const float2 k01 = h2f2(kv.x), k23 = h2f2(kv.y), k45 = h2f2(kv.z), k67 = h2f2(kv.w);
#pragma unroll
                    for (int h = 0; h < kAttnGroup; ++h) {
                        const float4 qa = *reinterpret_cast<const float4 *>(&qs[h][8 * i]);
                        const float4 qb = *reinterpret_cast<const float4 *>(&qs[h][8 * i + 4]);
                        s2[h].x = fmaf(k01.x, qa.x, s2[h].x);
                        s2[h].y = fmaf(k01.y, qa.y, s2[h].y);
                        s2[h].x = fmaf(k23.x, qa.z, s2[h].x);
                        s2[h].y = fmaf(k23.y, qa.w, s2[h].y);
                        s2[h].x = fmaf(k45.x, qb.x, s2[h].x);
                        s2[h].y = fmaf(k45.y, qb.y, s2[h].y);
                        s2[h].x = fmaf(k67.x, qb.z, s2[h].x);
                        s2[h].y = fmaf(k67.y, qb.w, s2[h].y);
                    }
                }
            }
#pragma unroll
            for (int h = 0; h < kAttnGroup; ++h) sc[h] = valid ? (s2[h].x + s2[h].y) * p.scale : -INFINITY;
        }
        float pr[kAttnGroup];
#pragma unroll
        for (int h = 0; h < kAttnGroup; ++h) {
            float cm = sc[h];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, o));
            const float mn = fmaxf(m[h], cm);  // finite: every chunk holds a valid key
            const float alpha = m[h] == -INFINITY ? 0.0f : expf(m[h] - mn);
            pr[h] = valid ? expf(sc[h] - mn) : 0.0f;
            float ps = pr[h];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
            l[h] = l[h] * alpha + ps;
            m[h] = mn;
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[h][j] *= alpha;
        }
        // P.V in batches of 8 keys, the batch's V loads issued before its arithmetic
        for (int j0 = 0; j0 < nvalid; j0 += 8) {
            uint2 vv[8];
#pragma unroll
            for (int u = 0; u < 8; ++u)
                vv[u] = j0 + u < nvalid
                            ? __ldg(reinterpret_cast<const uint2 *>(vh + (long)(base + j0 + u) * kAttnHeadDim) + lane)
                            : make_uint2(0u, 0u);
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const float2 v01 = h2f2(vv[u].x), v23 = h2f2(vv[u].y);
#pragma unroll
                for (int h = 0; h < kAttnGroup; ++h) {
                    const float pj = __shfl_sync(0xffffffffu, pr[h], (j0 + u) & 31);  // 0 past nvalid
                    acc[h][0] = fmaf(pj, v01.x, acc[h][0]);
                    acc[h][1] = fmaf(pj, v01.y, acc[h][1]);
                    acc[h][2] = fmaf(pj, v23.x, acc[h][2]);
                    acc[h][3] = fmaf(pj, v23.y, acc[h][3]);
                }
            }
        }
    }
    // merge the 4 warps: each publishes (m, l, acc), thread d combines dim d of every head
    if (lane == 0) {
#pragma unroll
        for (int h = 0; h < kAttnGroup; ++h) {
            wm[warp][h] = m[h];
            wl[warp][h] = l[h];
        }
    }
#pragma unroll
    for (int h = 0; h < kAttnGroup; ++h)
        *reinterpret_cast<float4 *>(&wacc[warp][h][4 * lane]) = make_float4(acc[h][0], acc[h][1], acc[h][2], acc[h][3]);
    __syncthreads();
    const int d = tid;  // 128 threads = 128 dims
#pragma unroll
    for (int h = 0; h < kAttnGroup; ++h) {
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < 4; ++w) M = fmaxf(M, wm[w][h]);
        float L = 0.0f, A = 0.0f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < 4; ++w) {
                if (wm[w][h] == -INFINITY) continue;
                const float e = expf(wm[w][h] - M);
                L = fmaf(wl[w][h], e, L);
                A = fmaf(wacc[w][h][d], e, A);
            }
        }
        float *rec = p.partials + ((long)split * p.query_heads + g * kAttnGroup + h) * kAttnPartial;
        if (d == 0) {
            rec[0] = M == -INFINITY ? -FLT_MAX : M;
            rec[1] = L;
        }
        rec[2 + d] = A;
    }
}

// Merge of the splits (gqa_combine_f16_128, decode_attention.cu:791-843): weights
// exp(max_s - max) for splits with a non-zero sum, output = sum_s w_s v_s / sum_s w_s l_s.
__global__ void __launch_bounds__(128) gqa_combine_kernel(const float *__restrict__ partials, __half *__restrict__ out,
                                                          int num_splits, int query_heads) {
    __shared__ float wts[kAttnMaxSplits];
    __shared__ float den;
    const int qh = blockIdx.x, d = threadIdx.x;
    const float *base = partials + (long)qh * kAttnPartial;
    const long stride = (long)query_heads * kAttnPartial;
    float M = -FLT_MAX;
    for (int s = 0; s < num_splits; ++s) M = fmaxf(M, base[s * stride]);
    if (d < num_splits) {
        const float *rec = base + d * stride;
        wts[d] = rec[1] == 0.0f ? 0.0f : expf(rec[0] - M);
    }
    __syncthreads();
    if (d == 0) {
        float t = 0.0f;
        for (int s = 0; s < num_splits; ++s) t = fmaf(base[s * stride + 1], wts[s], t);
        den = t;
    }
    __syncthreads();
    float v = 0.0f;
    for (int s = 0; s < num_splits; ++s) v = fmaf(base[s * stride + 2 + d], wts[s], v);
    out[(long)qh * kAttnHeadDim + d] = __float2half_rn(__fdiv_rn(v, den));
}

// Q8_1 blocks of num_rows rows (mmvq_gguf.cu:1137-1169): warp per 32-block.
__global__ void __launch_bounds__(256) quantize_q8_1_rows_kernel(const float *__restrict__ x, uint8_t *__restrict__ vy,
                                                                 int kx, int kx_padded, int num_rows) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const int nb = kx_padded / 32;
    if (warp >= nb * num_rows) return;
    const int row = warp / nb, b = warp % nb, i = b * 32 + lane;
    const float v = i < kx ? x[(long)row * kx + i] : 0.0f;
    float d, sum;
    const int8_t q = q81_lane(v, d, sum);
    uint8_t *blk = vy + ((long)row * nb + b) * 36;
    blk[4 + lane] = (uint8_t)q;
    if (lane == 0) {
        *reinterpret_cast<__half *>(blk) = __float2half_rn(d);
        *reinterpret_cast<__half *>(blk + 2) = __float2half_rn(sum);
    }
}

static int rope_launch(const RopeParams &r, cudaStream_t s) {
    if (r.q_rows < 0 || r.k_rows < 0 || r.head_dim <= 0 || r.rope_dim < 0 || r.rope_dim > r.head_dim ||
        r.rope_dim % 2 || r.position < 0 || (r.q_rows && !r.q) || (r.k_rows && !r.k) || (r.rope_dim && (!r.cos || !r.sin)))
        return MMRS_ERR_ARG;
    const int total = r.q_rows + (r.v ? 2 : 1) * r.k_rows;
    if (total == 0) return MMRS_OK;
    partial_rope_kernel<<<(total + 255) / 256, 256, 0, s>>>(r);
    return cudaGetLastError() == cudaSuccess ? MMRS_OK : MMRS_ERR_LAUNCH;
}

static int gqa_launch(const GqaParams &g, int kv_heads, __half *out, cudaStream_t s) {
    if (!g.q || !g.k || !g.v || !g.partials || !out || g.seq_len < 1 || g.num_splits < 1 ||
        g.num_splits > kAttnMaxSplits || kv_heads < 1 || g.query_heads != kAttnGroup * kv_heads ||
        g.q_head_stride < kAttnHeadDim || g.k_head_stride < (long)g.seq_len * kAttnHeadDim ||
        g.v_head_stride < (long)g.seq_len * kAttnHeadDim || ((uintptr_t)g.k & 15u) || ((uintptr_t)g.v & 15u) ||
        (g.k_head_stride % 8) || (g.v_head_stride % 8))
        return MMRS_ERR_ARG;
    gqa_decode_kernel<<<dim3(g.num_splits, kv_heads), 128, 0, s>>>(g);
    gqa_combine_kernel<<<g.query_heads, 128, 0, s>>>(g.partials, out, g.num_splits, g.query_heads);
    return cudaGetLastError() == cudaSuccess ? MMRS_OK : MMRS_ERR_LAUNCH;
}

static int qkv_launch(const void *x, void *vy, const void *vq, const void *vk, const void *vv, float *proj, int kx,
                      int kx_padded, int q_rows, int k_rows, int v_rows, cudaStream_t s) {
    if (!x || q_rows < 0 || k_rows < 0 || v_rows < 0) return MMRS_ERR_ARG;
    MvParams p = {};
    p.w[0] = static_cast<const uint8_t *>(vq);
    p.w[1] = static_cast<const uint8_t *>(vk);
    p.w[2] = static_cast<const uint8_t *>(vv);
    p.n[0] = q_rows;
    p.n[1] = k_rows;
    p.n[2] = v_rows;
    p.k = kx;
    p.kpad = kx_padded;
    p.x = x;
    p.vy_out = static_cast<uint8_t *>(vy);
    p.dst = proj;
    return mv_launch<float>(p, s);
}

// Row RMSNorm of the hidden state (candle-nn RmsNorm, src/model.rs:198-210: attn_norm / ffn_norm):
// y = x / sqrt(mean(x^2) + eps) * w, one CTA per row, fixed reduction order.
__global__ void __launch_bounds__(1024) rmsnorm_rows_kernel(const float *__restrict__ x, const float *__restrict__ w,
                                                            float *__restrict__ y, int n, float eps) {
    __shared__ float ws[32];
    const float *xr = x + (long)blockIdx.x * n;
    float *yr = y + (long)blockIdx.x * n;
    float ss = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) ss = fmaf(xr[i], xr[i], ss);
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, m);
    if ((threadIdx.x & 31) == 0) ws[threadIdx.x >> 5] = ss;
    __syncthreads();
    float t = (int)(threadIdx.x & 31) < (int)(blockDim.x >> 5) ? ws[threadIdx.x & 31] : 0.0f;
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) t += __shfl_xor_sync(0xffffffffu, t, m);
    const float scale = rsqrtf(__fdiv_rn(t, (float)n) + eps);
    for (int i = threadIdx.x; i < n; i += blockDim.x) yr[i] = __fmul_rn(__fmul_rn(xr[i], scale), w[i]);
}

}  // namespace mmrs

using namespace mmrs;

extern "C" int mmrs_rmsnorm_f32(const float *x, const float *weight, float *y, int n, int rows, float eps,
                                mmrs_stream_t stream) {
    if (!x || !weight || !y || n <= 0 || rows <= 0) return MMRS_ERR_ARG;
    rmsnorm_rows_kernel<<<rows, 1024, 0, (cudaStream_t)stream>>>(x, weight, y, n, eps);
    return cudaGetLastError() == cudaSuccess ? MMRS_OK : MMRS_ERR_LAUNCH;
}

// ------------------------------------------------------------------------------------------
// C ABI
// ------------------------------------------------------------------------------------------
extern "C" void launch_mmvq_gguf_quantize_q8_1_f32(const void *x, void *vy, int kx, int kx_padded, int num_rows,
                                                   void *stream) {
    if (!x || !vy || kx <= 0 || kx_padded < kx || kx_padded % 32 || num_rows <= 0) {
        record_error(MMRS_ERR_ARG);
        return;
    }
    const long warps = (long)(kx_padded / 32) * num_rows;
    quantize_q8_1_rows_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
        static_cast<const float *>(x), static_cast<uint8_t *>(vy), kx, kx_padded, num_rows);
    record_error(cudaGetLastError() == cudaSuccess ? MMRS_OK : MMRS_ERR_LAUNCH);
}

extern "C" void launch_mmvq_gguf_q8_0_f32_plain(const void *vx, const void *vy, void *dst, int ncols_x, int nrows_x,
                                                int stride_col_y, int stride_col_dst, int b_size, void *stream) {
    (void)stride_col_dst;  // one column: its stride does not matter
    if (b_size != 1) {
        record_error(MMRS_ERR_UNSUPPORTED);
        return;
    }
    if (!vx || !vy || !dst || nrows_x <= 0 || stride_col_y * 32 < ncols_x) {
        record_error(MMRS_ERR_ARG);
        return;
    }
    MvParams p = {};
    p.w[0] = static_cast<const uint8_t *>(vx);
    p.n[0] = nrows_x;
    p.k = ncols_x;
    p.kpad = stride_col_y * 32;
    p.vy_in = static_cast<const uint8_t *>(vy);
    p.dst = static_cast<float *>(dst);
    record_error(mv_launch<float>(p, (cudaStream_t)stream));
}

extern "C" void launch_mmvq_gguf_qkv_q8_0_f32(const void *x, void *vy, const void *vq, const void *vk, const void *vv,
                                             void *dst, int kx, int kx_padded, int q_rows, int k_rows, int v_rows,
                                             void *stream) {
    record_error(qkv_launch(x, vy, vq, vk, vv, static_cast<float *>(dst), kx, kx_padded, q_rows, k_rows, v_rows,
                            (cudaStream_t)stream));
}

extern "C" void launch_mmvq_gguf_qkv_q8_0_f32_rmsnorm_f16(const void *x, void *vy, const void *vq, const void *vk,
                                                         const void *vv, void *projection_dst, const void *q_alpha,
                                                         const void *k_alpha, void *dst, int kx, int kx_padded,
                                                         int q_rows, int k_rows, int v_rows, float eps, void *stream) {
    cudaStream_t s = (cudaStream_t)stream;
    if (!projection_dst || !dst || !q_alpha || !k_alpha) {
        record_error(MMRS_ERR_ARG);
        return;
    }
    int rc = qkv_launch(x, vy, vq, vk, vv, static_cast<float *>(projection_dst), kx, kx_padded, q_rows, k_rows,
                        v_rows, s);
    if (rc == MMRS_OK) {
        qkv_rmsnorm_f16_kernel<<<3, 1024, 0, s>>>(static_cast<const float *>(projection_dst),
                                                  static_cast<const float *>(q_alpha),
                                                  static_cast<const float *>(k_alpha), static_cast<__half *>(dst),
                                                  q_rows, k_rows, v_rows, eps);
        rc = cudaGetLastError() == cudaSuccess ? MMRS_OK : MMRS_ERR_LAUNCH;
    }
    record_error(rc);
}

extern "C" void launch_partial_rope_f16(const void *q, const void *k, const void *cos, const void *sin, void *dst,
                                        int q_rows, int k_rows, int head_dim, int rope_dim, int position,
                                        void *stream) {
    if (!dst) {
        record_error(MMRS_ERR_ARG);
        return;
    }
    RopeParams r = {};
    r.q = static_cast<const __half *>(q);
    r.k = static_cast<const __half *>(k);
    r.cos = static_cast<const float *>(cos);
    r.sin = static_cast<const float *>(sin);
    r.q_out = static_cast<__half *>(dst);
    r.k_out = static_cast<__half *>(dst) + q_rows;
    r.q_rows = q_rows;
    r.k_rows = k_rows;
    r.head_dim = head_dim;
    r.rope_dim = rope_dim;
    r.position = position;
    r.kv_stride = head_dim;
    record_error(rope_launch(r, (cudaStream_t)stream));
}

extern "C" void launch_gqa_decode_mma_f16_128(const void *q, const void *k, const void *v, void *partials,
                                              void *output, int seq_len, int q_head_stride, int k_head_stride,
                                              int v_head_stride, int num_splits, int query_heads, int kv_heads,
                                              float scale, int device_ordinal, void *stream) {
    (void)device_ordinal;  // no per-device kernel configuration is needed here
    GqaParams g = {};
    g.q = static_cast<const __half *>(q);
    g.k = static_cast<const __half *>(k);
    g.v = static_cast<const __half *>(v);
    g.partials = static_cast<float *>(partials);
    g.seq_len = seq_len;
    g.q_head_stride = q_head_stride;
    g.k_head_stride = k_head_stride;
    g.v_head_stride = v_head_stride;
    g.num_splits = num_splits;
    g.query_heads = query_heads;
    g.scale = scale;
    record_error(gqa_launch(g, kv_heads, static_cast<__half *>(output), (cudaStream_t)stream));
}

// ------------------------------------------------------------------------------------------
// Fused single-token attention half (Attention::forward, src/model.rs:79-162, T = 1).
// ------------------------------------------------------------------------------------------
namespace {
struct AttnLayout {
    size_t proj, qkv, qrot, part, out, total;
};
AttnLayout attn_layout(const MmrsAttnWeights *w) {
    const size_t qr = (size_t)w->query_heads * kAttnHeadDim, kr = (size_t)w->kv_heads * kAttnHeadDim;
    AttnLayout l{};
    size_t o = 0;
    auto take = [&](size_t b) {
        const size_t at = o;
        o = (o + b + 255) / 256 * 256;
        return at;
    };
    l.proj = take(sizeof(float) * (qr + 2 * kr));
    l.qkv = take(sizeof(__half) * (qr + 2 * kr));
    l.qrot = take(sizeof(__half) * qr);
    l.part = take(sizeof(float) * kAttnMaxSplits * w->query_heads * kAttnPartial);
    l.out = take(sizeof(__half) * qr);
    l.total = o;
    return l;
}
int attn_validate(const MmrsAttnWeights *w) {
    if (!w || !w->wq || !w->wk || !w->wv || !w->wo || !w->q_norm || !w->k_norm || !w->rope_cos || !w->rope_sin)
        return MMRS_ERR_ARG;
    if (w->hidden <= 0 || w->hidden % 64 || w->kv_heads < 1 || w->query_heads != kAttnGroup * w->kv_heads ||
        w->rope_dim < 0 || w->rope_dim > kAttnHeadDim || w->rope_dim % 2 || w->max_positions < 1)
        return MMRS_ERR_UNSUPPORTED;
    return MMRS_OK;
}
}  // namespace

extern "C" size_t mmrs_attn_workspace_bytes(const MmrsAttnWeights *w) {
    return attn_validate(w) == MMRS_OK ? attn_layout(w).total : 0;
}

extern "C" int mmrs_attn_decode_forward(const MmrsAttnWeights *w, const float *x, const float *residual, int position,
                                        void *k_cache, void *v_cache, float *y, void *workspace,
                                        size_t workspace_bytes, mmrs_stream_t stream) {
    int rc = attn_validate(w);
    if (rc != MMRS_OK) return rc;
    if (!x || !k_cache || !v_cache || !y || !workspace || position < 0 || position >= w->max_positions)
        return MMRS_ERR_ARG;
    const AttnLayout l = attn_layout(w);
    if (workspace_bytes < l.total || ((uintptr_t)workspace & 255u) || ((uintptr_t)k_cache & 15u) ||
        ((uintptr_t)v_cache & 15u))
        return MMRS_ERR_ARG;
    cudaStream_t s = (cudaStream_t)stream;
    uint8_t *ws = static_cast<uint8_t *>(workspace);
    float *proj = reinterpret_cast<float *>(ws + l.proj);
    __half *qkv = reinterpret_cast<__half *>(ws + l.qkv), *qrot = reinterpret_cast<__half *>(ws + l.qrot);
    __half *att = reinterpret_cast<__half *>(ws + l.out);
    const int qr = w->query_heads * kAttnHeadDim, kr = w->kv_heads * kAttnHeadDim;
    const long head_stride = (long)w->max_positions * kAttnHeadDim;
    // 1. Q / K / V projection (one launch for the three matrices) and Q / K RMSNorm to f16
    rc = qkv_launch(x, nullptr, w->wq, w->wk, w->wv, proj, w->hidden, w->hidden, qr, kr, kr, s);
    if (rc != MMRS_OK) return rc;
    qkv_rmsnorm_f16_kernel<<<3, 1024, 0, s>>>(proj, w->q_norm, w->k_norm, qkv, qr, kr, kr, w->eps);
    // 2. rotary embedding of Q (into qrot) and K, K and V appended to the caches at `position`
    RopeParams r = {};
    r.q = qkv;
    r.k = qkv + qr;
    r.v = qkv + qr + kr;
    r.cos = w->rope_cos;
    r.sin = w->rope_sin;
    r.q_out = qrot;
    r.k_out = static_cast<__half *>(k_cache) + (long)position * kAttnHeadDim;
    r.v_out = static_cast<__half *>(v_cache) + (long)position * kAttnHeadDim;
    r.q_rows = qr;
    r.k_rows = kr;
    r.head_dim = kAttnHeadDim;
    r.rope_dim = w->rope_dim;
    r.position = position;
    r.kv_stride = head_stride;
    rc = rope_launch(r, s);
    if (rc != MMRS_OK) return rc;
    // 3. attention over positions [0, position]: splits of 128 keys (one 32-key chunk per warp)
    const int seq = position + 1;
    const int splits = std::max(1, std::min((seq + 127) / 128, kAttnMaxSplits));
    GqaParams g = {};
    g.q = qrot;
    g.k = static_cast<const __half *>(k_cache);
    g.v = static_cast<const __half *>(v_cache);
    g.partials = reinterpret_cast<float *>(ws + l.part);
    g.seq_len = seq;
    g.q_head_stride = kAttnHeadDim;
    g.k_head_stride = head_stride;
    g.v_head_stride = head_stride;
    g.num_splits = splits;
    g.query_heads = w->query_heads;
    g.scale = 1.0f / sqrtf((float)kAttnHeadDim);
    rc = gqa_launch(g, w->kv_heads, att, s);
    if (rc != MMRS_OK) return rc;
    // 4. output projection of the f16 attention output (+ residual)
    MvParams o = {};
    o.w[0] = static_cast<const uint8_t *>(w->wo);
    o.n[0] = w->hidden;
    o.k = qr;
    o.kpad = qr;
    o.x = att;
    o.residual = residual;
    o.dst = y;
    return mv_launch<__half>(o, s);
}
