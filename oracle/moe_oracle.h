/*
 * CPU oracle for the MiniMax-M2.7 sparse-MoE hot path — TEST INFRASTRUCTURE ONLY.
 *
 * This is a plain-C restatement of the reference's arithmetic for the MoE block over GGUF
 * k-quant experts (spmurrayzzz/minimax-rs, vendored Candle kernels).  It exists to check the
 * CUDA product path and to time the CPU baseline.  Only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline / reference arm may load it; the product library never links it.
 *
 * Every function cites the reference file:line it follows (paths relative to the reference
 * project root).  The parity pins for this oracle are listed in tests/golden/README.md.
 */
#ifndef MINIMAX_MOE_ORACLE_H
#define MINIMAX_MOE_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ORC_QK_K 256
#define ORC_QK8_1 32
#define ORC_Q4K_BYTES 144 /* half2 dm + 12 scale bytes + 128 nibble bytes (gguf.cuh:341-344) */
#define ORC_Q5K_BYTES 176 /* half2 dm + 12 scale bytes + 32 qh + 128 qs (gguf.cuh:382-386) */
#define ORC_Q81_BYTES 36  /* half2 ds + 32 int8 (gguf.cuh:401-406) */

/* GGUF type codes used on the reference FFI (candle-nn/src/moe.rs:293-306). */
enum { ORC_Q8_0 = 0, ORC_Q4K = 1, ORC_Q2K = 2, ORC_Q3K = 3, ORC_Q5K = 4, ORC_Q6K = 5 };

/* ---- scalar helpers ---------------------------------------------------------------- */
float orc_half_to_float(uint16_t h);
uint16_t orc_float_to_half(float f); /* IEEE binary16, round to nearest even */
size_t orc_row_bytes(int gguf_type, int k);

/* ---- dequantisation (candle-kernels/src/quantized.cu:925-1010) -------------------- */
/* fused=1: y = fmaf(d*sc, q, -(dmin*m)) (one rounding); fused=0: (d*sc)*q - dmin*m.   */
void orc_dequant_q4k(const uint8_t *blocks, int64_t nblocks, float *out, int fused);
void orc_dequant_q5k(const uint8_t *blocks, int64_t nblocks, float *out, int fused);

/* ---- activation quantisation ------------------------------------------------------- */
/* Decode/generic Q8_1 (moe/gguf.cuh:1234-1261): d = amax/127, q = roundf(x/d),
 * ds = half2(d, warp-butterfly sum).  out: rows x (kpad/32) blocks of 36 bytes. */
void orc_quantize_q8_1(const float *x, int rows, int k, int kpad, uint8_t *out);
/* MMQ DS4 Q8_1 (mmq_gguf/mmq_quantize.cu:11-107): d_inv = 127/amax, q = roundf(x*d_inv),
 * ds = half2(1/d_inv, sum).  Logical layout: q[rows][kpad], d/s[rows][kpad/32] half bits.
 * src_rows (nullable) gathers row i from x[src_rows[i]]. */
void orc_quantize_q8_1_mmq(const float *x, const int32_t *src_rows, int rows, int k, int kpad,
                           int8_t *q, uint16_t *d, uint16_t *s);

/* ---- row dot products -------------------------------------------------------------- */
/* MMVQ formula (moe/gguf.cuh:727-750, 783-813, 1038-1170). */
float orc_dot_q4k_q81(const uint8_t *wrow, const uint8_t *q81row, int nsb);
float orc_dot_q5k_q81(const uint8_t *wrow, const uint8_t *q81row, int nsb);
/* MMQ MMA formula (mmq_gguf/mmq_gguf.cuh:2050-2150 tile load, :1170-1230 combine). */
float orc_dot_kq_mmq(int gguf_type, const uint8_t *wrow, const int8_t *q, const uint16_t *d,
                     const uint16_t *s, int nsb);

/* ---- routing ------------------------------------------------------------------------ */
/* Router logits in the library's canonical summation order: K cut into 8 slices; per slice 32
 * lane partials (lane l accumulates float4 groups l, l+32, ... with fmaf) summed by xor-butterfly
 * 16,8,4,2,1; slice sums added as ((s0+s1)+(s2+s3))+((s4+s5)+(s6+s7)).  K % 32 == 0. */
void orc_router_logits(const float *x, const float *wr, int T, int E, int K, float *logits);
/* fused_moe.rs:228-241 + moe_gguf.cu:47-76: s = 1/(1+expf(-l)); select top-k of s+bias
 * (ties: lower id first); w = s[id]/tree-sum (fixed +4,+2,+1 order for topk=8). */
void orc_route_topk(const float *logits, const float *bias, int T, int E, int topk,
                    uint32_t *topk_ids, float *topk_w);
/* minimax_moe_decode_topk (moe_gguf.cu:34-100): adds the expert-sorted (expert, route) pair. */
void orc_decode_topk(const float *logits, const float *bias, uint32_t *topk_ids, float *topk_w,
                     uint32_t *expert_ids, uint32_t *route_ids);
/* moe_sort_routes (moe_sort.cu:21-51): stable sort of route ids by expert id. */
void orc_sort_routes(const uint32_t *expert_ids, int n, uint32_t *sorted_experts,
                     uint32_t *sorted_routes);

/* ---- expert GEMMs on the reference FFI semantics ------------------------------------ */
/* moe_gemm_gguf (moe_gguf.cu:127-196, 357-424). */
void orc_moe_gemm_gguf(const float *input, const uint8_t *weights, const int32_t *sorted_token_ids,
                       const int32_t *expert_ids, const float *topk_weights, float *output,
                       int num_experts, int topk, int size_m, int size_n, int size_k,
                       int gguf_type);
/* moe_gemm_mmq_gguf (mmq_moe.cu:69-165). */
void orc_moe_gemm_mmq(const float *input, const uint8_t *weights, const int32_t *sorted_token_ids,
                      const int32_t *expert_ids, const float *topk_weights, float *output,
                      int num_experts, int topk, int size_m, int size_n, int size_k,
                      int gguf_type);
/* moe_gemm_gguf_decode_silu (moe_gguf.cu:200-343, 426-567). */
void orc_moe_decode_silu(const float *input, const uint8_t *gate_w, const uint8_t *up_w,
                         const uint8_t *down_w, const int32_t *sorted_token_ids,
                         const int32_t *expert_ids, const float *topk_weights, float *output,
                         int num_experts, int topk, int hidden, int inter, int gate_up_type,
                         int down_type);

/* ---- the MoE block (FusedMoeGGUF::forward, fused_moe.rs:251-334) -------------------- */
typedef struct {
    const float *router;   /* [E][H] f32 */
    const float *bias;     /* [E] f32 (e_score_correction_bias) */
    const uint8_t *gate;   /* [E][I][H] GGUF blocks */
    const uint8_t *up;     /* [E][I][H] */
    const uint8_t *down;   /* [E][H][I] */
    int gate_up_type, down_type;
    int num_experts, topk, hidden, inter;
} OrcMoeWeights;

/* y[T][H] = MoE(x[T][H]) (+ residual if non-null).  Dispatch mirrors the reference:
 * T==1 -> fused decode; 2<=T<mmq_min -> generic GEMV; T>=mmq_min -> MMQ numerics.
 * topk_ids/topk_w (nullable) receive the routing.  Threads: OpenMP, all available. */
void orc_moe_block(const OrcMoeWeights *w, const float *x, const float *residual, int T,
                   int mmq_min_tokens, float *y, uint32_t *topk_ids, float *topk_w);

/* Number of OpenMP threads the oracle uses (for the CPU-baseline report). */
int orc_num_threads(void);
void orc_set_threads(int n);

/* ---- decode attention (attn_oracle.c) ---- */
uint16_t orc_double_to_half(double v);
void orc_q8_0_matvec(const uint8_t *w, int rows, int k, const float *x, float *y);

/* ---- LM head (lmhead_oracle.c) ---- */
void orc_q6k_dequant_row(const uint8_t *row, int k, float *out);
void orc_q6k_matvec(const uint8_t *w, int rows, int k, const float *x, float *y);
int orc_argmax_f32(const float *v, int n);
void orc_qkv_rmsnorm_f16(const float *proj, const float *q_alpha, const float *k_alpha, int q_rows,
                         int k_rows, int v_rows, float eps, uint16_t *dst);
void orc_partial_rope_f16(const uint16_t *q, const uint16_t *k, const float *cosv, const float *sinv, int q_rows,
                          int k_rows, int head_dim, int rope_dim, int position, uint16_t *dst);
void orc_gqa_decode_f16(const uint16_t *q, const uint16_t *k, const uint16_t *v, int seq_len, int q_heads,
                        int kv_heads, int head_dim, int64_t kv_head_stride, float scale, uint16_t *out);

/* ---- token sampling (sample_oracle.c); statuses as the CUDA path's ---- */
#define MMRS_ERR_ARG_ORC 1
#define MMRS_ERR_NONFINITE_ORC 7
int orc_sample_token(const float *logits, int vocab, double temperature, double top_p, int top_k, double u,
                     int32_t *token, double *margin);
int orc_token_logprob(const float *logits, int vocab, int token_id, float *out);

#ifdef __cplusplus
}
#endif
#endif
