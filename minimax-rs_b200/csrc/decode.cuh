// Parameters of the fused single-token MoE kernel (decode.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace mmrs {

struct GridFlags;

struct DecodeParams {
    const float *x;       // [H] f32
    const float *router;  // [E][H] f32 (internal routing only)
    const float *bias;    // [E] f32 (internal routing only)
    const uint8_t *gate;  // [E][I][H] GGUF
    const uint8_t *up;    // [E][I][H]
    const uint8_t *down;  // [E][H][I]
    const float *residual;  // [H] or null
    float *y;               // [H]
    uint32_t *topk_ids_out;  // [8] or null
    float *topk_w_out;       // [8] or null
    // external routing (moe_gemm_gguf_decode_silu): pairs in expert order, weights by route
    const int32_t *ext_route;
    const int32_t *ext_expert;
    const float *ext_w;
    int internal_routing;
    // workspace
    float *logits;        // [E]
    float *act;           // [8][I] f32 up * silu(gate)
    int8_t *aq;           // [8][I] Q8_1 quants of act
    float *ad;            // [8][I/32] fp16-rounded Q8_1 scales
    int *aS;              // [8][I/32] sums of quants
    uint32_t *blk_count;  // [8][I/32] (unused by the current kernel; kept in the layout)
    GridFlags *ctl;
    uint64_t *trace;  // [grid][16] globaltimer stamps per phase, or null
    // shape
    int E, H, I;
    int gu_type, dn_type;
    // launch configuration (decode_configure): lanes per row, rows per sub-unit (one warp's
    // share) and rows per copy unit (one ring stage) of the gate/up and down matrices
    int gu_lanes, gu_sub_rows, gu_unit_rows, dn_lanes, dn_sub_rows, stages, stage_bytes, grid;
    int act_slots, res_slots;
    uint64_t timeout_ns;
    // multi-GPU group (world > 1): this rank's exchange region and every rank's as mapped here;
    // ep = 1: only experts e with e % world == rank are computed on this rank
    uint8_t *xch;
    const uint8_t *xpeer[8];
    int world, rank, ep;
    // operation token of the group (monotonic, the same on every rank, never 0): the exchange
    // flags and double-buffered partial rows belong to the group, not to a layer's workspace
    uint32_t token;
};

size_t decode_smem_bytes(const DecodeParams &p);
int decode_configure(DecodeParams &p, int num_sms, int max_smem);
int decode_launch(const DecodeParams &p, cudaStream_t stream);

}  // namespace mmrs
