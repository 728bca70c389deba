// Tensor-parallel Q/K RMSNorm of a decode step (TP = 2) on B200 (sm_100a).
//
// MiniMax-M2.7 normalises Q and K over their full width (all 48 query heads, all 8 KV heads), so
// with heads split across ranks every rank needs the sum of squares of the other rank's part.
// The reference (src/tensor_parallel_model.rs:123-139, 142-168, 407-419) runs per rank: the Q8_0
// QKV matvec (launch_mmvq_gguf_qkv_q8_0_f32), the rank-local sums (launch_qkv_tp_sumsq_f32), a
// two-float all-reduce over the peer link (launch_tp2_peer_all_reduce_f32 with count 2), and the
// normalisation + partial RoPE + f16 conversion with the global sums
// (launch_qkv_tp_rmsnorm_rope_f16).  The two launchers here take the reference's names and
// arguments.
//   sums:  one CTA per projection (Q, K), 1024 threads; thread t adds columns t, t + 1024, ... in
//          f32 (fused multiply-add), then a 32-lane butterfly, the 32 warp sums in shared memory and one more
//          butterfly: the reference's summation order, so the statistics (and everything after
//          them) are bit-identical to the reference's.
//   norm:  one thread per output element: scale = rsqrt(global / full_rows + eps); the element
//          (scale * x * alpha, rounded to half) is rotated against its pair in the first rope_dim
//          columns of its head with the arithmetic of launch_partial_rope_f16; V is converted.
// Both are tiny (a few thousand elements) and latency-bound; they sit between the projection and
// the attention kernel on each rank.
#include <cuda_fp16.h>

#include "../../include/minimax_attn.h"
#include "common.cuh"
#include "workspace.cuh"

namespace mmrs {
namespace {

constexpr int kSsThreads = 1024;

__global__ void __launch_bounds__(kSsThreads) qkv_tp_sumsq_kernel(const float *q, const float *k, float *stats,
                                                                  int q_rows, int k_rows) {
    const int which = blockIdx.x, tid = threadIdx.x;
    const float *src = which == 0 ? q : k;
    const int n = which == 0 ? q_rows : k_rows;
    float acc = 0.0f;
    for (int c = tid; c < n; c += kSsThreads) {
        const float v = src[c];
        acc = fmaf(v, v, acc);  // the reference's `sum += value * value` as compiled (contracted)
    }
    acc = warp_sum_butterfly(acc);
    __shared__ float per_warp[32];
    if ((tid & 31) == 0) per_warp[tid >> 5] = acc;
    __syncthreads();
    if (tid < 32) {
        const float w = warp_sum_butterfly(per_warp[tid]);
        if (tid == 0) stats[which] = w;
    }
}

struct TpNormParams {
    const float *q, *k, *v, *stats, *q_alpha, *k_alpha, *cos, *sin;
    __half *dst;
    int q_rows, k_rows, v_rows, q_full, k_full, head_dim, rope_dim, position;
    float eps;
};

__device__ __forceinline__ __half tp_scaled(const float *src, const float *alpha, int i, float scale) {
    return __float2half_rn(__fmul_rn(__fmul_rn(scale, src[i]), alpha[i]));
}

__global__ void __launch_bounds__(256) qkv_tp_rmsnorm_rope_kernel(const TpNormParams p) {
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    const int qk = p.q_rows + p.k_rows;
    if (idx >= qk + p.v_rows) return;
    if (idx >= qk) {
        p.dst[idx] = __float2half_rn(p.v[idx - qk]);
        return;
    }
    const bool is_q = idx < p.q_rows;
    const int local = is_q ? idx : idx - p.q_rows;
    const float *src = is_q ? p.q : p.k;
    const float *alpha = is_q ? p.q_alpha : p.k_alpha;
    const float scale = rsqrtf(__fadd_rn(__fdiv_rn(p.stats[is_q ? 0 : 1], (float)(is_q ? p.q_full : p.k_full)), p.eps));
    const __half x = tp_scaled(src, alpha, local, scale);
    const int col = local % p.head_dim;
    if (col >= p.rope_dim) {
        p.dst[idx] = x;
        return;
    }
    const int half_rope = p.rope_dim / 2;
    const bool first = col < half_rope;
    const int pair = first ? local + half_rope : local - half_rope;
    const int freq = first ? col : col - half_rope;
    const __half xp = tp_scaled(src, alpha, pair, scale);
    const __half c = __float2half_rn(p.cos[p.position * half_rope + freq]);
    const __half sn = __float2half_rn(p.sin[p.position * half_rope + freq]);
    p.dst[idx] = first ? __hfma(x, c, __hneg(__hmul_rn(xp, sn))) : __hfma(xp, sn, __hmul_rn(x, c));
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
    if (!q || !k || !v || !global_stats || !q_alpha || !k_alpha || !cos || !sin || !dst || q_rows < 0 ||
        k_rows < 0 || v_rows < 0 || head_dim <= 0 || rope_dim < 0 || rope_dim > head_dim || (rope_dim & 1) ||
        q_rows % head_dim || k_rows % head_dim || q_full_rows <= 0 || k_full_rows <= 0 || position < 0) {
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
    const int total = q_rows + k_rows + v_rows;
    if (total > 0) qkv_tp_rmsnorm_rope_kernel<<<(total + 255) / 256, 256, 0, (cudaStream_t)stream>>>(p);
    record_error(cudaGetLastError() == cudaSuccess ? MMRS_OK : MMRS_ERR_LAUNCH);
}
