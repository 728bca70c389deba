/*
 * minimax_moe.h — C ABI of the B200-native MiniMax-M2.7 sparse-MoE hot path.
 *
 * Two groups of entry points:
 *
 *  1. Drop-in replacements for the reference's launchers.  Names, argument order and meaning
 *     follow the reference's Rust FFI declarations (vendor/candle-kernels/src/ffi.rs) so that the
 *     reference's `extern "C"` block links against this library unchanged.  Like the reference
 *     they return void; host-side validation failures and launch errors are recorded in a
 *     thread-local status readable with mmrs_last_error().  Device pointers and a CUDA stream
 *     (passed as a handle, `i64` / `*mut c_void` on the Rust side) are the only arguments.
 *
 *  2. New fused entry points (prefix mmrs_) that return an int status (MMRS_OK == 0).
 *
 * All buffers are device memory owned by the caller unless stated otherwise.  Expert weights
 * are raw GGUF block bytes laid out [experts][rows][k/256 blocks], rows contiguous (the layout
 * of the reference's QTensor storage), 16-byte aligned.
 */
#ifndef MINIMAX_MOE_H
#define MINIMAX_MOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *mmrs_stream_t; /* == cudaStream_t */

#if defined(__GNUC__)
#define MMRS_API __attribute__((visibility("default")))
#else
#define MMRS_API
#endif

/* ---- status codes ------------------------------------------------------------------- */
#define MMRS_OK 0
#define MMRS_ERR_ARG 1         /* invalid shape, pointer, alignment or enum                  */
#define MMRS_ERR_UNSUPPORTED 2 /* GGUF type or shape this build does not implement          */
#define MMRS_ERR_LAUNCH 3      /* CUDA launch / runtime error                                 */
#define MMRS_ERR_TIMEOUT 4     /* a bounded device-side wait (grid barrier, peer flag) expired */
#define MMRS_ERR_ALLOC 5       /* device allocation failed                                    */
#define MMRS_ERR_SCRATCH_LIMIT 6 /* problem larger than the fixed scratch of                  */
                                 /* mmrs_moe_block_decode_static                              */

/* ---- GGUF type codes (candle-nn/src/moe.rs:293-306) ---------------------------------- */
#define MMRS_Q8_0 0
#define MMRS_Q4K 1
#define MMRS_Q2K 2
#define MMRS_Q3K 3
#define MMRS_Q5K 4
#define MMRS_Q6K 5

/* ===================================================================================== */
/* 1. Reference launchers (vendor/candle-kernels/src/ffi.rs)                              */
/* ===================================================================================== */

/* ffi.rs:41-49 — replaces moe_gguf.cu:94-100 (minimax_moe_decode_topk_kernel).
 * logits[256], bias[256] f32 -> sigmoid, top-8 of sigmoid+bias, renormalised weights, plus the
 * expert-id-sorted (expert_ids, route_ids) pair consumed by the decode MoE kernels. */
MMRS_API void minimax_moe_decode_topk(const float *logits, const float *bias, uint32_t *topk_ids,
                             float *topk_weights, uint32_t *expert_ids, uint32_t *route_ids,
                             mmrs_stream_t stream);

/* ffi.rs:51-67 — replaces moe_gguf.cu:426-567 (moe_gemm_gguf_decode_silu).
 * One token, topk == 8: y[hidden] = sum_k w_k * down_k(silu(gate_k x) * up_k x).
 * sorted_token_ids / expert_ids are the (route, expert) pairs in expert order; topk_weights is
 * indexed by route.  Types: gate/up Q4_K or Q5_K, down Q4_K or Q5_K. */
MMRS_API void moe_gemm_gguf_decode_silu(const float *input, const void *gate_weights,
                               const void *up_weights, const void *down_weights,
                               const int32_t *sorted_token_ids, const int32_t *expert_ids,
                               const float *topk_weights, float *output, int num_experts,
                               int topk, int hidden_size, int intermediate_size,
                               int gate_up_gguf_dtype, int down_gguf_dtype, mmrs_stream_t stream);

/* ffi.rs:25-39 — replaces moe_gguf.cu:357-424 (moe_gemm_gguf, the generic path for T < 32).
 * output[route][size_n] = W[expert] . q8_1(input[row]) for every (route, expert) pair of the
 * expert-sorted lists sorted_token_ids / expert_ids (size_m entries).  Input row = route / topk
 * when topk_weights is NULL (gate / up), else route, and the row is scaled by
 * topk_weights[route] (down).  Q8_1 as quantize_q8_1 (d = amax/127, q = round(x/d)).
 * Types: Q4_K, Q5_K (others: MMRS_ERR_UNSUPPORTED, nothing launched). */
MMRS_API void moe_gemm_gguf(const float *input, const void *weights, const int32_t *sorted_token_ids,
                            const int32_t *expert_ids, const float *topk_weights, float *output,
                            int num_experts, int topk, int size_m, int size_n, int size_k,
                            int gguf_dtype, mmrs_stream_t stream);

/* ffi.rs:86-100 — replaces mmq_gguf/mmq_moe.cu:69-165 (moe_gemm_mmq_gguf, T >= 32).
 * Same contract as moe_gemm_gguf with the MMQ numerics: quantize_mmq_q8_1<DS4>
 * (d_inv = 127/amax, q = round(x*d_inv)) and the per-32-block combine dmA.x*d8*C + dmA.y*s8.
 * Types other than Q4_K / Q5_K do nothing (as the reference) and record MMRS_ERR_UNSUPPORTED. */
MMRS_API void moe_gemm_mmq_gguf(const float *input, const void *weights,
                                const int32_t *sorted_token_ids, const int32_t *expert_ids,
                                const float *topk_weights, float *output, int num_experts, int topk,
                                int size_m, int size_n, int size_k, int gguf_dtype,
                                mmrs_stream_t stream);

/* ffi.rs:102-109 — replaces moe/moe_sort.cu:21-51 (CUB radix sort of (key, route) pairs).
 * Stable sort of size keys on bits [0, end_bit): expert_ids_sorted receives the keys,
 * route_ids_sorted the original positions.  end_bit <= 10 (MMRS_ERR_UNSUPPORTED beyond). */
MMRS_API void moe_sort_routes(const uint32_t *expert_ids_unsorted, uint32_t *expert_ids_sorted,
                              uint32_t *route_ids_sorted, int size, int end_bit,
                              mmrs_stream_t stream);

/* Status of the last reference-ABI call made by this host thread (MMRS_OK when it launched). */
MMRS_API int mmrs_last_error(void);

/* ===================================================================================== */
/* 2. Fused MoE block                                                                     */
/* ===================================================================================== */

/* Weights of one MoE layer (one rank's shard under tensor parallelism).  Mirrors the fields of
 * FusedMoeGGUF (vendor/candle-transformers/src/fused_moe.rs:162-175). */
typedef struct {
    const float *router; /* [num_experts][hidden] f32 (ffn_gate_inp, dequantised)        */
    const float *bias;   /* [num_experts] f32 (exp_probs_b, e_score_correction_bias)     */
    const void *gate;    /* [num_experts][inter][hidden] GGUF blocks                     */
    const void *up;      /* [num_experts][inter][hidden]                                 */
    const void *down;    /* [num_experts][hidden][inter]                                 */
    int gate_up_type;    /* MMRS_Q4K or MMRS_Q5K                                          */
    int down_type;       /* MMRS_Q4K or MMRS_Q5K                                          */
    int num_experts;     /* 256 for MiniMax-M2.7                                          */
    int topk;            /* 8                                                             */
    int hidden;          /* 3072 (multiple of 256)                                        */
    int inter;           /* 1536, or 768 per rank at TP=2 (multiple of 256)               */
} MmrsMoeWeights;

/* Device workspace the block needs for up to max_tokens tokens.  Its first
 * mmrs_moe_workspace_zero_bytes(w) bytes (status word, launch tags, tagged routing logits, phase
 * trace and the tagged activation records the CTAs exchange) must be zero before first use;
 * mmrs_moe_workspace_status() clears them again after a call that reported MMRS_ERR_TIMEOUT.
 * Launches that share a workspace must be ordered on one stream. */
MMRS_API size_t mmrs_moe_workspace_bytes(const MmrsMoeWeights *w, int max_tokens);
MMRS_API size_t mmrs_moe_workspace_zero_bytes(const MmrsMoeWeights *w);

/* y[T][hidden] = MoE(x[T][hidden]) (+ residual[T][hidden] when non-null), f32.
 * Replaces FusedMoeGGUF::forward (fused_moe.rs:251-334) + the residual add of
 * Layer::forward (src/model.rs:213-218).  topk_ids [T][topk] / topk_weights [T][topk]
 * (nullable) receive the routing.  T == 1 runs the fused decode kernel; T > 1 runs routing,
 * stable bucketing, gathered Q8_1 and the grouped tensor-core expert GEMMs (MMQ numerics for
 * T >= 32, the generic ones below, as fused_moe.rs:296-316).  x, y, residual 16-byte aligned. */
MMRS_API int mmrs_moe_block_forward(const MmrsMoeWeights *w, const float *x, const float *residual,
                           float *y, int num_tokens, uint32_t *topk_ids, float *topk_weights,
                           void *workspace, size_t workspace_bytes, mmrs_stream_t stream);

/* No counterpart in the reference (its MoE input already lives on the device).  The same block
 * as mmrs_moe_block_forward for a caller holding x and y in host memory, num_tokens * hidden
 * floats each way, enqueued on `stream` in one call.  Pinned (mapped) host buffers are read by a
 * small kernel into x_dev and written by the block's final stores directly; other host buffers
 * go through copy-engine transfers via x_dev / y_dev.  residual, topk_ids and topk_weights are
 * device pointers as in mmrs_moe_block_forward; x_dev / y_dev 16-byte aligned. */
MMRS_API int mmrs_moe_block_forward_host(const MmrsMoeWeights *w, const float *x_host, const float *residual,
                                         float *y_host, int num_tokens, float *x_dev, float *y_dev,
                                         uint32_t *topk_ids, float *topk_weights, void *workspace,
                                         size_t workspace_bytes, mmrs_stream_t stream);

/* Copies the per-CTA phase timestamps (globaltimer ns, 32 slots per CTA: 0 start, 1 router done,
 * 2 routing candidates ready, 3 copy table done, 4 gate/up done, 5 activation records read,
 * 6 activation scales built, 7 end, 8 first weight copy issued, 9 last copy issued, 10 first
 * down copy issued, 11 own activation blocks published, 12 x quantised, 13 routing warp 0's
 * candidates written, 14 slots and weights merged, 15 copy table computed, 16 weighted expert
 * rows summed, 17 thread 0's down dots done, 18 multi-GPU rows pushed, 19 routing lane 0's
 * score seen, 20 slots merged, 21 thread 0's first activation block begun, 22 own activation
 * blocks published (thread 0), 23 its act values formed, 24 + w routing warp w's candidates
 * written) of the
 * last single-token launch into host_out.  Returns the number of entries copied, or -status. */
MMRS_API int mmrs_moe_workspace_trace(const void *workspace, uint64_t *host_out, int max_entries,
                                      mmrs_stream_t stream);

/* No counterpart in the reference.  Same single-token block as mmrs_moe_block_forward with
 * num_tokens == 1, for callers that cannot allocate device memory when they call it: an engine
 * whose device memory is fully pre-reserved by its own allocator, or a call site that, like the
 * reference's FFI, passes only tensor pointers and has no workspace to hand over.  It allocates
 * nothing: its scratch is a fixed 128 KiB device array inside this library, held by every GPU
 * that loads the library until the process exits.
 * Limits: num_experts <= 256, inter <= 1536, hidden <= 3072; larger problems return
 * MMRS_ERR_SCRATCH_LIMIT without launching.  The first call on a device resolves the array's
 * device address and caches it, so make that first call before any stream capture.  All calls
 * on a device share the array; each clears the part that must start at zero on `stream`, so
 * calls that overlap on the GPU (unordered streams or host threads) race. */
MMRS_API int mmrs_moe_block_decode_static(const MmrsMoeWeights *w, const float *x,
                                          const float *residual, float *y, uint32_t *topk_ids,
                                          float *topk_weights, mmrs_stream_t stream);

/* No counterpart in the reference.  Device-side status of the last mmrs_moe_block_decode_static
 * call on the current device: synchronises `stream`, returns MMRS_OK or MMRS_ERR_TIMEOUT (a
 * bounded wait of that call expired and y was not written) and clears the word.  Allocates
 * nothing.  The next static call clears the word as well, so read it before that call.  The
 * cached scratch address is tied to the device's current context: do not call the static entry
 * points across a cudaDeviceReset in the same process. */
MMRS_API int mmrs_moe_static_status(mmrs_stream_t stream);

/* Reads back (synchronising `stream`) and clears the device-side status word of a workspace. */
MMRS_API int mmrs_moe_workspace_status(void *workspace, mmrs_stream_t stream);

/* ===================================================================================== */
/* 2b. Multi-GPU: tensor parallel (TP=2, the reference layout) and expert parallel (W=4/8)  */
/* ===================================================================================== */

/* Reference two-rank peer collectives (ffi.rs:505-528; mmvq_gguf.cu:888-966).
 * launch_tp2_peer_all_reduce_f32: output = local + peer (+ residual); with normalized_output,
 * normalized_output = output * rsqrt(mean(output^2) + eps) * norm_weight.  Both ranks launch with
 * the same epoch (0: self counter in self_signal[2]).  Signal buffers are 128-byte peer-visible
 * words, zero before first use; waits are bounded (2 s) and an expiry sets self_signal[3] to
 * MMRS_ERR_TIMEOUT.  Launch status: mmrs_last_error(). */
MMRS_API void launch_tp2_peer_all_reduce_f32(const void *local, const void *peer, const void *residual,
                                             const void *norm_weight, void *output,
                                             void *normalized_output, void *self_signal,
                                             void *peer_signal, unsigned int epoch, int count,
                                             float norm_eps, void *stream);
MMRS_API void launch_tp2_peer_broadcast_f32(const void *source, void *output, void *self_signal,
                                            void *peer_signal, unsigned int epoch, int rank,
                                            int count, void *stream);

/* No counterpart struct in the reference (it passes peer pointers per call).  One rank's view of
 * a group of `world` GPUs.  `mine` is this rank's exchange region (mmrs_peer_alloc of
 * mmrs_xch_bytes(ar_capacity) bytes, zeroed); peers[r] is rank r's region as mapped in this
 * process (CUDA IPC between processes, or plain device pointers with peer access inside one
 * process), read-write: the single-token exchange stores this rank's rows into every peer's
 * region; peers[rank] == mine.  expert_parallel = 0: tensor parallel, every rank holds
 * gate/up rows [rank * inter, (rank + 1) * inter) and the matching down K range of every expert
 * (MmrsMoeWeights.inter is the per-rank inter); 1: expert parallel, rank r holds the full
 * experts e with e % world == r (MmrsMoeWeights still points at [num_experts] tensors; the
 * non-owned experts' bytes are never read). */
typedef struct {
    int world;
    int rank;
    void *mine;
    void *peers[8];
    size_t ar_capacity; /* floats per all-reduce buffer: >= T * hidden of the largest T > 1 call */
    int expert_parallel;
} MmrsPeerGroup;

MMRS_API size_t mmrs_xch_bytes(size_t ar_capacity);
MMRS_API int mmrs_peer_alloc(size_t bytes, void **ptr);       /* cudaMalloc + zero */
MMRS_API int mmrs_peer_free(void *ptr);
MMRS_API int mmrs_ipc_handle(void *ptr, uint8_t *handle64);    /* 64-byte CUDA IPC handle */
MMRS_API int mmrs_ipc_open(const uint8_t *handle64, void **ptr);
MMRS_API int mmrs_ipc_close(void *ptr);
MMRS_API int mmrs_peer_enable(int peer_device);                /* one process, several GPUs */

/* Multi-rank all-reduce of partial vectors: every rank writes its partial [count] f32 into
 * mmrs_xch_ar_buffer(g, token) (earlier on `stream`), then all ranks call mmrs_peer_all_reduce
 * with the same token (monotonic, starting at 1): y = sum over ranks in rank order (+ residual),
 * bit-identical on all ranks.  count <= ar_capacity. */
MMRS_API float *mmrs_xch_ar_buffer(const MmrsPeerGroup *g, uint32_t token);
MMRS_API int mmrs_peer_all_reduce(const MmrsPeerGroup *g, const float *residual, float *y,
                                  size_t count, uint32_t token, mmrs_stream_t stream);
/* Reads back (synchronising `stream`) and clears the group's device status word. */
MMRS_API int mmrs_peer_status(const MmrsPeerGroup *g, mmrs_stream_t stream);

/* The MoE block on one rank of a group (replaces the TP rank worker's MoE call plus
 * TensorParallelRankGroup::all_reduce_sum_with_residual, tensor_parallel.rs:786-812): y is the
 * full block output (+ residual) on every rank.  T == 1: the fused decode kernel exchanges the
 * ranks' partial rows over NVLink inside the same launch.  T > 1: the multi-token path on the
 * rank's shard, then mmrs_peer_all_reduce.  `token` is the group's operation counter for every T:
 * the same value on all ranks, monotonic over all calls on the group (whatever the layer), never
 * 0 (MMRS_ERR_ARG).  The exchange flags and partial buffers belong to the group, so layers that
 * share a group must not reuse tokens. */
MMRS_API int mmrs_moe_block_forward_group(const MmrsMoeWeights *w, const MmrsPeerGroup *g,
                                          const float *x, const float *residual, float *y,
                                          int num_tokens, uint32_t *topk_ids, float *topk_weights,
                                          void *workspace, size_t workspace_bytes, uint32_t token,
                                          mmrs_stream_t stream);

/* No counterpart in the reference.  mmrs_moe_block_forward_group for a rank holding x and y in
 * host memory, num_tokens * hidden floats each way, enqueued on `stream` in one call, as
 * mmrs_moe_block_forward_host does on one GPU: pinned (mapped) host buffers are read by a small
 * kernel into x_dev and written by the group's final stores directly; other host buffers go
 * through copy-engine transfers via x_dev / y_dev.  Same token rules as the device form. */
MMRS_API int mmrs_moe_block_forward_group_host(const MmrsMoeWeights *w, const MmrsPeerGroup *g,
                                               const float *x_host, const float *residual, float *y_host,
                                               int num_tokens, float *x_dev, float *y_dev, uint32_t *topk_ids,
                                               float *topk_weights, void *workspace, size_t workspace_bytes,
                                               uint32_t token, mmrs_stream_t stream);

/* ===================================================================================== */
/* 3. Seeded synthetic data (bench / test inputs; same generator as the numpy mirror)     */
/* ===================================================================================== */

/* dst[i] = scale * N(0,1)_i (Irwin-Hall(8) of 16-bit uniforms from a counter-based SplitMix64
 * stream), optionally rounded to bf16 (stored as f32). */
MMRS_API int mmrs_synth_normal_f32(float *dst, int64_t n, uint64_t seed, uint32_t stream_id, float scale,
                          int round_bf16, mmrs_stream_t stream);

/* Writes the [row0, row0+nrows) x [kblk0, kblk0+nkblk) window of a synthetic k-quant tensor of
 * shape [experts][rows][k/256 blocks] into dst (laid out [experts][nrows][nkblk]).  Every byte is
 * uniform except each block's half2 (d, dmin) = fp16(|N(0,1)| * 0.01). */
MMRS_API int mmrs_synth_kquant(void *dst, int gguf_type, uint64_t seed, uint32_t stream_id, int experts,
                      int rows, int k, int row0, int nrows, int kblk0, int nkblk,
                      mmrs_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* MINIMAX_MOE_H */
