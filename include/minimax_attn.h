/*
 * minimax_attn.h — C ABI of the single-token (decode) attention half of a MiniMax-M2.7 layer on
 * B200: Q8_0 Q/K/V projection with Q/K RMSNorm, partial rotary embedding, split-K GQA decode
 * attention over an f16 KV cache, and the Q8_0 output projection.
 *
 * Reference-named entry points follow vendor/candle-kernels/src/ffi.rs (names, argument order and
 * meaning; void return, failures recorded for mmrs_last_error()).  Pointers are device memory; the
 * stream is a cudaStream_t handle.  Q8_0 matrices are raw GGUF blocks (half d, 32 int8: 34 bytes)
 * laid out [rows][k/32], 4-byte aligned, with k a multiple of 64.  Fixed head geometry of the
 * attention kernels: head_dim 128, 6 query heads per KV head (the reference's kernels are built
 * for the same shapes).
 */
#ifndef MINIMAX_ATTN_H
#define MINIMAX_ATTN_H

#include "minimax_moe.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ---- drop-ins for the reference's launchers ------------------------------------------- */

/* ffi.rs:465-471 (mmvq_gguf.cu:1296-1307): x f32 [num_rows][kx] -> Q8_1 blocks vy
 * [num_rows][kx_padded / 32] (36 bytes: half d = amax / 127, half sum, 32 int8; zero past kx). */
MMRS_API void launch_mmvq_gguf_quantize_q8_1_f32(const void *x, void *vy, int kx, int kx_padded, int num_rows,
                                                 void *stream);

/* ffi.rs:270-280 (mmvq_gguf.cu:1173-1200, q8_0 / f32 instance): dst[col * stride_col_dst + row] =
 * Q8_0 row `row` of vx dotted with Q8_1 column `col` of vy (stride_col_y blocks per column),
 * for b_size columns.  This build implements b_size == 1. */
MMRS_API void launch_mmvq_gguf_q8_0_f32_plain(const void *vx, const void *vy, void *dst, int ncols_x, int nrows_x,
                                              int stride_col_y, int stride_col_dst, int b_size, void *stream);

/* ffi.rs:473-486 (mmvq_gguf.cu:1309-1323): quantise x f32 [kx] into vy, then dst f32
 * [q_rows + k_rows + v_rows] = [Wq x | Wk x | Wv x] for Q8_0 vq, vk, vv. */
MMRS_API void launch_mmvq_gguf_qkv_q8_0_f32(const void *x, void *vy, const void *vq, const void *vk, const void *vv,
                                           void *dst, int kx, int kx_padded, int q_rows, int k_rows, int v_rows,
                                           void *stream);

/* ffi.rs:487-503 (mmvq_gguf.cu:1325-1336): the projection above into projection_dst, then dst
 * f16 = [RMSNorm(q) * q_alpha | RMSNorm(k) * k_alpha | v] (RMSNorm over all q_rows / k_rows). */
MMRS_API void launch_mmvq_gguf_qkv_q8_0_f32_rmsnorm_f16(const void *x, void *vy, const void *vq, const void *vk,
                                                       const void *vv, void *projection_dst, const void *q_alpha,
                                                       const void *k_alpha, void *dst, int kx, int kx_padded,
                                                       int q_rows, int k_rows, int v_rows, float eps, void *stream);

/* ffi.rs:529-536 (mmvq_gguf.cu:970-990, 1360-1366): tensor-parallel decode, before the Q/K
 * statistics all-reduce: stats[0] = sum of q[i]^2 over this rank's q_rows, stats[1] = the same over
 * k (f32, the reference's summation order: bit-identical statistics). */
MMRS_API void launch_qkv_tp_sumsq_f32(const void *q, const void *k, void *stats, int q_rows, int k_rows,
                                      void *stream);

/* ffi.rs:537-557 (mmvq_gguf.cu:995-1034, 1368-1382): after the all-reduce, dst f16
 * [q_rows + k_rows + v_rows] = [rope(RMSNorm_global(q) * q_alpha) | rope(RMSNorm_global(k) * k_alpha)
 * | v]: scale = rsqrt(global_stats[0 or 1] / q_full_rows (k_full_rows) + eps) over the full,
 * all-rank width; the first rope_dim columns of every head_dim-wide head rotated by the f32 tables
 * cos / sin [positions][rope_dim / 2] at `position`, with launch_partial_rope_f16's arithmetic. */
MMRS_API void launch_qkv_tp_rmsnorm_rope_f16(const void *q, const void *k, const void *v, const void *global_stats,
                                             const void *q_alpha, const void *k_alpha, const void *cos,
                                             const void *sin, void *dst, int q_rows, int k_rows, int v_rows,
                                             int q_full_rows, int k_full_rows, int head_dim, int rope_dim,
                                             int position, float eps, void *stream);

/* ffi.rs:558-570 (mmvq_gguf.cu:1038-1066, 1385-1395): dst f16 [q_rows + k_rows] = q, k (f16) with
 * the first rope_dim columns of every head_dim-wide head rotated by the f32 tables
 * cos / sin [positions][rope_dim / 2] at `position`. */
MMRS_API void launch_partial_rope_f16(const void *q, const void *k, const void *cos, const void *sin, void *dst,
                                      int q_rows, int k_rows, int head_dim, int rope_dim, int position,
                                      void *stream);

/* ffi.rs:571-587 (decode_attention.cu:845-918): single-token GQA over seq_len cached positions.
 * q f16 [query_heads][q_head_stride]; k, v f16, KV head g at g * k_head_stride (v_head_stride),
 * position t at + t * 128; partials f32 [num_splits][query_heads][130] (max, sum, 128 values)
 * scratch; output f16 [query_heads][128].  query_heads == 6 * kv_heads, 1 <= num_splits <= 128. */
MMRS_API void launch_gqa_decode_mma_f16_128(const void *q, const void *k, const void *v, void *partials, void *output,
                                            int seq_len, int q_head_stride, int k_head_stride, int v_head_stride,
                                            int num_splits, int query_heads, int kv_heads, float scale,
                                            int device_ordinal, void *stream);

/* No counterpart as a launcher in the reference (candle-nn RmsNorm, used for attn_norm / ffn_norm,
 * src/model.rs:198-210): y[r] = x[r] / sqrt(mean(x[r]^2) + eps) * weight for `rows` rows of n
 * floats.  Returns an MMRS status. */
MMRS_API int mmrs_rmsnorm_f32(const float *x, const float *weight, float *y, int n, int rows, float eps,
                              mmrs_stream_t stream);

/* ---- fused single-token attention half of a layer --------------------------------------- */

typedef struct {
    const void *wq, *wk, *wv; /* Q8_0 [q_rows][hidden], [k_rows][hidden], [k_rows][hidden]   */
    const void *wo;           /* Q8_0 [hidden][q_rows]                                         */
    const float *q_norm;      /* f32 [q_rows]  (attn_q_norm)                                   */
    const float *k_norm;      /* f32 [k_rows]  (attn_k_norm)                                   */
    const float *rope_cos;    /* f32 [max_positions][rope_dim / 2]                             */
    const float *rope_sin;
    int hidden;               /* 3072                                                          */
    int query_heads;          /* 48                                                            */
    int kv_heads;             /* 8                                                             */
    int rope_dim;             /* 64                                                            */
    int max_positions;        /* rows of the rotary tables and KV cache capacity              */
    float eps;                /* RMSNorm epsilon (1e-6)                                        */
} MmrsAttnWeights;

/* Workspace bytes of mmrs_attn_decode_forward (caller-owned, 256-byte aligned, zero before first
 * use: it holds per-KV-head split counters that every call leaves at zero, and a status word). */
MMRS_API size_t mmrs_attn_workspace_bytes(const MmrsAttnWeights *w);

/* Status word of a workspace after its calls completed (synchronous read): MMRS_OK, or
 * MMRS_ERR_TIMEOUT when a bounded wait inside the attention kernel expired. */
MMRS_API int mmrs_attn_workspace_status(const void *workspace);

/* No single counterpart in the reference: Attention::forward for one token (src/model.rs:79-162)
 * as one call.  x f32 [hidden] (the attn_norm output); the token's rotated K and its V are
 * written into the f16 caches k_cache / v_cache [kv_heads][max_positions][128] at `position`,
 * then the query attends to positions [0, position]; y f32 [hidden] = Wo . attention (+ residual
 * when given).  Returns an MMRS status. */
MMRS_API int mmrs_attn_decode_forward(const MmrsAttnWeights *w, const float *x, const float *residual, int position,
                                      void *k_cache, void *v_cache, float *y, void *workspace,
                                      size_t workspace_bytes, mmrs_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* MINIMAX_ATTN_H */
