// Parameters of the fused single-token MoE kernel (decode.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace mmrs {

// Control block of the single-token kernel at the start of its workspace.  Launch n (n = 1, 2,
// ...) of a workspace carries the tag n, and everything one CTA hands to the others travels in
// 64-bit words {tag, payload} written and read with relaxed stores and loads: a reader that sees
// the current tag sees the current payload, with no fence.  The routing lanes poll the score
// words directly.  For the activation records, each CTA adds 1 (relaxed) to a counter after
// writing its words, which reaches G * n in launch n: one thread per CTA waits for that, then the
// CTA reads the words (coalesced), re-reading any whose tag is not yet current.
//   n_act       the activation exchange counter (on its own 128-byte line);
//   arrive[c]   the tag of CTA c's last launch (its launch count; read only by CTA c);
// The sigmoid of the router logit of expert e (payload: the f32 bits) is published by the CTA
// that computed the logit into every one of kScoreReplicas copies of the score array (workspace,
// after the trace); CTA c polls copy c % kScoreReplicas, so each line is polled by a few CTAs
// instead of all of them.
//   zero_bytes  the size of the workspace prefix that must be zero before first use (control
//               block, trace and the tagged activation records), for the status reset.
constexpr int kDecodeMaxCtas = 256;
// globaltimer stamps a CTA records per launch (trace slots, see the phase list in decode.cu)
constexpr int kTraceSlots = 32;
constexpr int kScoreReplicas = 16;
struct DecodeCtl {
    uint32_t status;  // MMRS_OK, or MMRS_ERR_TIMEOUT once any wait expired
    uint32_t zero_bytes;
    uint32_t pad0[30];
    uint32_t n_act;
    uint32_t pad2[31];
    uint32_t arrive[kDecodeMaxCtas];
};

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
    unsigned long long *arec;  // [8 I / 32][9] tagged Q8_1 records of act: quants 4j..4j+3 (word
                               // j < 8), {fp16 scale, int16 sum of quants} (word 8)
    uint32_t zero_bytes;       // workspace prefix that must start at zero
    DecodeCtl *ctl;
    uint64_t *trace;  // [grid][kTraceSlots] globaltimer stamps per phase, or null
    unsigned long long *score;  // [kScoreReplicas][256] tagged sigmoids of the router logits
    // shape
    int E, H, I;
    int gu_type, dn_type;
    // launch configuration (decode_configure): rows per gate/up copy unit, ring stages and their
    // size, grid (one CTA per SM)
    int gu_unit_rows, stages, stage_bytes, grid;
    int act_slots, res_slots;
    uint64_t timeout_ns;
    // multi-GPU group (world > 1): this rank's exchange region and every rank's as mapped here;
    // ep = 1: only experts e with e % world == rank are computed on this rank
    uint8_t *xch;
    uint8_t *xpeer[8];  // peer-mapped regions (the decode kernel stores its rows into them)
    int world, rank, ep;
    // operation token of the group (monotonic, the same on every rank, never 0): the exchange
    // flags and double-buffered partial rows belong to the group, not to a layer's workspace
    uint32_t token;
};

size_t decode_smem_bytes(const DecodeParams &p);
int decode_configure(DecodeParams &p, int num_sms, int max_smem);
int decode_launch(const DecodeParams &p, cudaStream_t stream);

}  // namespace mmrs
