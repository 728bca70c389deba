// Tensor-parallel Q/K RMSNorm of a decode step (TP = 2) on B200 (sm_100a).
//
// MiniMax-M2.7 normalises Q and K over their full width (all 48 query heads, all 8 KV heads), so
// with heads split across ranks every rank needs the other rank's sum of squares.  The reference
// (src/tensor_parallel_model.rs:123-139, 142-168, 407-419) runs per rank: the Q8_0 QKV matvec,
// the rank-local sums (launch_qkv_tp_sumsq_f32), a two-float all-reduce over the peer link
// (launch_tp2_peer_all_reduce_f32 with count 2), and the normalisation + partial RoPE + f16
// conversion with the global sums (launch_qkv_tp_rmsnorm_rope_f16).  The two launchers here keep
// the reference's names and arguments (drop-in); the statistics must be the reference's bit for
// bit, which fixes the summation order (1024 strided f32 partials, each a chain of fused
// multiply-adds over its columns in order, a 32-lane butterfly per 32 consecutive partials, and a
// butterfly over those 32 sums), not the launch shape:
//   sums:  one 256-thread CTA per projection; lane l of warp w carries the four partials
//          32 (w + 8 j) + l, j = 0..3 (four independent chains in flight per thread, coalesced
//          loads), butterflies them per j into shared memory in partial-group order, and warp 0
//          finishes with the butterfly over the 32 group sums.
//   norm:  one thread per column pair of a head: inside the rotated prefix a thread owns the
//          rotation pair (col f, col f + rope_dim / 2) and writes both rotated outputs (the
//          launch_partial_rope_f16 arithmetic); beyond it, two plain columns as one half2; V is
//          converted two values at a time.
#include <cuda_fp16.h>

#include "../../include/minimax_attn.h"
#include "common.cuh"
#include "workspace.cuh"

namespace mmrs {
namespace {

constexpr int kPartials = 1024;   // strided partial sums of the statistic (the order to reproduce)
constexpr int kSsWarps = 8;
constexpr int kSsThreads = 32 * kSsWarps;
constexpr int kPerLane = kPartials / kSsThreads;  // 4

__global__ void __launch_bounds__(kSsThreads) qkv_tp_sumsq_kernel(const float *q, const float *k, float *stats,
                                                                  int q_rows, int k_rows) {
    __shared__ float group_sum[kPartials / 32];
    const float *src = blockIdx.x == 0 ? q : k;
    const int n = blockIdx.x == 0 ? q_rows : k_rows;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float acc[kPerLane];
#pragma unroll
    for (int j = 0; j < kPerLane; ++j) acc[j] = 0.0f;
    // partial t = 32 (warp + 8 j) + lane sums columns t, t + 1024, ... in order
    for (int c0 = 0; c0 < n; c0 += kPartials) {
#pragma unroll
        for (int j = 0; j < kPerLane; ++j) {
            const int c = c0 + 32 * (warp + kSsWarps * j) + lane;
            if (c < n) {
                const float v = src[c];
                acc[j] = fmaf(v, v, acc[j]);  // the reference's `sum += value * value` as compiled
            }
        }
    }
#pragma unroll
    for (int j = 0; j < kPerLane; ++j) {
        const float g = warp_sum_butterfly(acc[j]);
        if (lane == 0) group_sum[warp + kSsWarps * j] = g;
    }
    __syncthreads();
    if (warp == 0) {
        const float total = warp_sum_butterfly(group_sum[lane]);
        if (lane == 0) stats[blockIdx.x] = total;
    }
}

struct TpNormParams {
    const float *q, *k, *v, *stats, *q_alpha, *k_alpha, *cos, *sin;
    __half *dst;
    int q_rows, k_rows, v_rows, q_full, k_full, head_dim, rope_dim, position;
    float eps;
};

// scale * x * alpha, rounded to half (the reference's order of the two products)
__device__ __forceinline__ __half tp_scaled(float x, float alpha, float scale) {
    return __float2half_rn(__fmul_rn(__fmul_rn(scale, x), alpha));
}

__global__ void __launch_bounds__(256) qkv_tp_rmsnorm_rope_kernel(const TpNormParams p) {
    const int item = blockIdx.x * blockDim.x + threadIdx.x;
    const int hp = p.head_dim / 2;  // column pairs of a head
    const int qk_items = (p.q_rows + p.k_rows) / 2;
    if (item >= qk_items) {
        const int vi = item - qk_items;  // V: two values per item (an odd count ends with one)
        const int e = 2 * vi;
        if (e + 1 < p.v_rows) {
            *reinterpret_cast<__half2 *>(p.dst + p.q_rows + p.k_rows + e) = __floats2half2_rn(p.v[e], p.v[e + 1]);
        } else if (e < p.v_rows) {
            p.dst[p.q_rows + p.k_rows + e] = __float2half_rn(p.v[e]);
        }
        return;
    }
    const bool is_q = item < p.q_rows / 2;
    const int li = is_q ? item : item - p.q_rows / 2;  // pair item within the projection
    const int head = li / hp, f = li % hp;
    const float *src = (is_q ? p.q : p.k) + head * p.head_dim;
    const float *alpha = (is_q ? p.q_alpha : p.k_alpha) + head * p.head_dim;
    __half *out = p.dst + (is_q ? 0 : p.q_rows) + head * p.head_dim;
    const float scale = rsqrtf(__fadd_rn(__fdiv_rn(p.stats[is_q ? 0 : 1], (float)(is_q ? p.q_full : p.k_full)), p.eps));
    const int half_rope = p.rope_dim / 2;
    if (f < half_rope) {
        // rotation pair (a = col f, b = col f + half_rope) at frequency f
        const __half a = tp_scaled(src[f], alpha[f], scale);
        const __half b = tp_scaled(src[f + half_rope], alpha[f + half_rope], scale);
        const __half c = __float2half_rn(p.cos[p.position * half_rope + f]);
        const __half sn = __float2half_rn(p.sin[p.position * half_rope + f]);
        out[f] = __hfma(a, c, __hneg(__hmul_rn(b, sn)));
        out[f + half_rope] = __hfma(a, sn, __hmul_rn(b, c));
        return;
    }
    // two plain columns beyond the rotated prefix
    const int col = p.rope_dim + 2 * (f - half_rope);
    if (col + 1 < p.head_dim) {
        const __half x0 = tp_scaled(src[col], alpha[col], scale), x1 = tp_scaled(src[col + 1], alpha[col + 1], scale);
        *reinterpret_cast<__half2 *>(out + col) = __halves2half2(x0, x1);
    } else if (col < p.head_dim) {
        out[col] = tp_scaled(src[col], alpha[col], scale);
    }
}

}  // namespace
}  // namespace mmrs

using namespace mmrs;

extern "C" void launch_qkv_tp_sumsq_f32(const void *q, const void *k, void *stats, int q_rows, int k_rows,
                                        void *stream) {
    if (!q || !k || !stats || q_rows < 0 || k_rows < 0) {
        record_error(MMRS_ERR_ARG);
        return;
    }
    qkv_tp_sumsq_kernel<<<2, kSsThreads, 0, (cudaStream_t)stream>>>(
        static_cast<const float *>(q), static_cast<const float *>(k), static_cast<float *>(stats), q_rows, k_rows);
    record_error(cudaGetLastError() == cudaSuccess ? MMRS_OK : MMRS_ERR_LAUNCH);
}

extern "C" void launch_qkv_tp_rmsnorm_rope_f16(const void *q, const void *k, const void *v, const void *global_stats,
                                               const void *q_alpha, const void *k_alpha, const void *cos,
                                               const void *sin, void *dst, int q_rows, int k_rows, int v_rows,
                                               int q_full_rows, int k_full_rows, int head_dim, int rope_dim,
                                               int position, float eps, void *stream) {
    // column pairs and half2 stores: even head_dim, even rope_dim <= head_dim
    if (!q || !k || !v || !global_stats || !q_alpha || !k_alpha || !cos || !sin || !dst || q_rows < 0 ||
        k_rows < 0 || v_rows < 0 || head_dim <= 0 || (head_dim & 1) || rope_dim < 0 || rope_dim > head_dim ||
        (rope_dim & 1) || q_rows % head_dim || k_rows % head_dim || q_full_rows <= 0 || k_full_rows <= 0 ||
        position < 0 || ((uintptr_t)dst & 3u)) {
        record_error(MMRS_ERR_ARG);
        return;
    }
    TpNormParams p = {};
    p.q = static_cast<const float *>(q);
    p.k = static_cast<const float *>(k);
    p.v = static_cast<const float *>(v);
    p.stats = static_cast<const float *>(global_stats);
    p.q_alpha = static_cast<const float *>(q_alpha);
    p.k_alpha = static_cast<const float *>(k_alpha);
    p.cos = static_cast<const float *>(cos);
    p.sin = static_cast<const float *>(sin);
    p.dst = static_cast<__half *>(dst);
    p.q_rows = q_rows;
    p.k_rows = k_rows;
    p.v_rows = v_rows;
    p.q_full = q_full_rows;
    p.k_full = k_full_rows;
    p.head_dim = head_dim;
    p.rope_dim = rope_dim;
    p.position = position;
    p.eps = eps;
    const int items = (q_rows + k_rows) / 2 + (v_rows + 1) / 2;
    if (items > 0) qkv_tp_rmsnorm_rope_kernel<<<(items + 255) / 256, 256, 0, (cudaStream_t)stream>>>(p);
    record_error(cudaGetLastError() == cudaSuccess ? MMRS_OK : MMRS_ERR_LAUNCH);
}
