/*
 * minimax_lmhead.h — C ABI of the output projection (LM head) of a MiniMax-M2.7 decode step on
 * B200: output_norm, the Q6_K `output` matrix against the final hidden state, greedy token.
 *
 * Reference-named entry point per vendor/candle-kernels/src/ffi.rs (name, argument order and
 * meaning; void return, failures recorded for mmrs_last_error()).  Pointers are device memory;
 * the stream is a cudaStream_t handle.  Q6_K matrices are raw GGUF blocks (ql[128], qh[64], int8
 * scales[16], half d: 210 bytes per 256 weights) laid out [rows][k/256], 16-byte aligned.
 */
#ifndef MINIMAX_LMHEAD_H
#define MINIMAX_LMHEAD_H

#include "minimax_moe.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ffi.rs:325-335 (mmvq_gguf.cu:609-632, 808-809, 1173-1200, q6_k / f32 instance): dst[row] =
 * Q6_K row `row` of vx dotted with the Q8_1 column vy (stride_col_y blocks per column, 16-byte
 * aligned), for b_size columns.  This build implements b_size == 1 and ncols_x a multiple of 256
 * up to 8192 (4, 8, 12 or 16 super-blocks). */
MMRS_API void launch_mmvq_gguf_q6_k_f32_plain(const void *vx, const void *vy, void *dst, int ncols_x, int nrows_x,
                                              int stride_col_y, int stride_col_dst, int b_size, void *stream);

typedef struct {
    const void *weight;        /* Q6_K [vocab][hidden] (`output.weight`)                      */
    const float *norm_weight;  /* f32 [hidden] (`output_norm.weight`), or null: no norm      */
    int vocab;                 /* 200064                                                       */
    int hidden;                /* 3072                                                         */
    float eps;                 /* RMSNorm epsilon (1e-6)                                       */
} MmrsLmHead;

/* Workspace bytes of mmrs_lm_head_forward (caller-owned, 256-byte aligned, zero before first use:
 * it holds the greedy choice's maximum and a CTA counter, both left zero by every call). */
MMRS_API size_t mmrs_lm_head_workspace_bytes(const MmrsLmHead *h);

/* Status word of a workspace after its calls completed (synchronous read): MMRS_OK, or
 * MMRS_ERR_TIMEOUT when a bounded wait expired. */
MMRS_API int mmrs_lm_head_workspace_status(const void *workspace);

/* No single counterpart in the reference: TensorParallelModel::logits for the last position
 * (src/tensor_parallel_model.rs:871-880) followed by greedy sampling (src/sampling.rs:84-88).
 * x f32 [hidden] (the final hidden state); logits f32 [vocab]; token (int32, device memory,
 * may be null) = the first index of the largest logit.  Returns an MMRS status. */
MMRS_API int mmrs_lm_head_forward(const MmrsLmHead *h, const float *x, float *logits, int32_t *token,
                                  void *workspace, size_t workspace_bytes, mmrs_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* MINIMAX_LMHEAD_H */
