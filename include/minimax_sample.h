/*
 * minimax_sample.h — C ABI of token sampling over a decode step's logits on B200: greedy,
 * top-k, top-p (nucleus) and temperature sampling, and the log-probability of one token, all on
 * the device that holds the logits (no vocabulary-sized copy to the host).
 *
 * Reference: src/sampling.rs (TokenSampler::sample, :84-150; exponential_weights, :161-177;
 * compare_candidates, :154-159; token_logprob, :60-75; SamplingParams::validate, :31-39).  The
 * reference draws its random number from a per-request StdRng (`rng.random::<f64>()`, one draw
 * per stochastic sample); here the caller keeps that generator and passes the draw as `u`, so
 * the GPU choice for a given draw is the reference's choice.
 *
 * Pointers are device memory; the stream is a cudaStream_t handle.  Status codes as in
 * minimax_moe.h.  The workspace is caller-owned, 256-byte aligned and zero before first use;
 * every completed call leaves it ready for the next one (a call that ended in MMRS_ERR_TIMEOUT
 * leaves it to be zeroed again).  One workspace serves one stream at a time.
 */
#ifndef MINIMAX_SAMPLE_H
#define MINIMAX_SAMPLE_H

#include "minimax_moe.h"

#ifdef __cplusplus
extern "C" {
#endif

#define MMRS_ERR_NONFINITE 7 /* logits (or the log-probability) not finite: no token written   */

/* SamplingParams (src/sampling.rs:13-17).  Valid: temperature finite and >= 0, top_p finite in
 * [0, 1] (validate, :31-39); top_k 0 = no top-k cut. */
typedef struct {
    double temperature;
    double top_p;
    int top_k;
} MmrsSamplingParams;

/* Largest vocabulary a call takes (token ids fit 20 bits). */
#define MMRS_SAMPLE_MAX_VOCAB 1048576
/* Largest candidate set that top-p sorts: min(top_k, vocab) when top_k > 0, else the nucleus
 * itself.  A larger nucleus ends in MMRS_ERR_UNSUPPORTED (device status, token -1). */
#define MMRS_SAMPLE_MAX_SORTED 1024

/* Workspace bytes of mmrs_sample_token / mmrs_token_logprob for this vocabulary (0: vocabulary
 * out of range). */
MMRS_API size_t mmrs_sample_workspace_bytes(int vocab);

/* Outcome of the last completed call on a workspace (synchronous read): MMRS_OK,
 * MMRS_ERR_NONFINITE, MMRS_ERR_UNSUPPORTED (nucleus over MMRS_SAMPLE_MAX_SORTED) or
 * MMRS_ERR_TIMEOUT (a grid barrier's bounded wait expired). */
MMRS_API int mmrs_sample_workspace_status(const void *workspace);

/* No single counterpart in the reference: TokenSampler::sample (src/sampling.rs:84-150) with the
 * draw `u` = rng.random::<f64>() in [0, 1) supplied by the caller.  logits f32 [vocab]; token
 * int32 (device memory) = the chosen id, or -1 when the device status is not MMRS_OK.
 *   temperature 0: the first index of the largest logit (logits.argmax, :87-89; no finiteness
 *     check, as the reference).
 *   otherwise: non-finite logits -> MMRS_ERR_NONFINITE (:97-99); candidates = the top_k largest
 *     (logit descending, then id ascending: compare_candidates); with top_p < 1 and more than one
 *     candidate, the sorted candidates are cut after the first whose cumulative weight
 *     exp(l - max) reaches top_p of the total (:110-125); then one candidate is drawn with weights
 *     exp((l - max) / temperature) by walking the cumulative weights against u * total (:127-150).
 *     Without the top-p cut the walk visits candidates by ascending id (the reference's order when
 *     top_k is 0 or >= vocab; for 0 < top_k < vocab the reference walks in the order its
 *     partial selection left, which no caller can observe except through the draw).
 * Host-side errors (MMRS_ERR_ARG: null pointers, vocab out of range, invalid params, u outside
 * [0, 1), short workspace) launch nothing. */
MMRS_API int mmrs_sample_token(const float *logits, int vocab, const MmrsSamplingParams *params, double u,
                               int32_t *token, void *workspace, size_t workspace_bytes, mmrs_stream_t stream);

/* token_logprob (src/sampling.rs:60-75): out (f32, device memory) = ln softmax(logits)[token_id]
 * over the unfiltered distribution, accumulated in double.  token_id >= vocab -> MMRS_ERR_ARG;
 * a non-finite result -> device status MMRS_ERR_NONFINITE. */
MMRS_API int mmrs_token_logprob(const float *logits, int vocab, int token_id, float *out, void *workspace,
                                size_t workspace_bytes, mmrs_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* MINIMAX_SAMPLE_H */
