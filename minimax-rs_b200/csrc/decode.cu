// Fused single-token MoE block for B200 (sm_100a).
//
// Replaces, in one persistent launch, the reference's decode chain
//   router Linear (fused_moe.rs:267) -> minimax_moe_decode_topk (moe_gguf.cu:34-100)
//   -> quantize_q8_1 -> moe_gate_up_decode_kernel -> quantize_silu_mul_q8_1
//   -> moe_down_decode_kernel (moe_gguf.cu:200-343, 426-567) -> + residual (model.rs:218)
//
// One CTA per SM: 12 consumer warps + 1 producer warp.  There is no grid barrier: what one CTA
// hands to the others travels in 64-bit words {launch tag, payload} in the workspace, written
// and read with relaxed accesses (a release fence costs ~0.6 us, more while copies stream), and
// a reader waits (bounded) until the words it needs carry this launch's tag.
//   P0  router GEMV in the canonical order (8 K-slices; the CTA's two experts x 8 slices are 16
//       (expert, slice) pairs over the 13 warps: 32 lane partials, butterfly, fixed slice tree).
//       The router rows are requested before anything else; the sigmoids of the two logits are
//       published tagged.
//   P1  eight consumer warps take 32 experts each (wait for the tagged sigmoid, order-preserving
//       selection key with the bias loaded at kernel start, rank among the warp's 32: that
//       warp's top-8), then rank their 8 candidates among all 64 (the global top-8) and quantise
//       their slice of x to Q8_1; the producer warp, which built the copy-table structure while
//       they waited, renormalises the weights and fills in the copy sources with its 32 lanes.
//   P2  gate/up: the CTA owns a contiguous range of (slot, row) pairs; copy units of rows of the
//       gate or the up matrix (one bulk copy each) stream through a ring of shared-memory stages.
//       Consumer lane t keeps the activation of x super-block t % (H/256) in registers for the
//       whole phase and computes that block of rows t / (H/256), + slots, ... in unit order; the
//       per-block partial sums go to shared memory.  Per unit, warp-aggregated counters find the
//       lane that completes it, which frees its stage and issues the unit `stages` later into it,
//       so the down units (this CTA's output rows of one expert: one contiguous copy each) land
//       in the ring while gate/up is still being computed.
//   P3  the CTA's gate/up range is a whole number of 32-row Q8_1 blocks, so it sums the block
//       partials, quantises act = up * silu(gate) of its own blocks (quantize_silu_mul_q8_1
//       arithmetic) and publishes each as nine tagged words; every CTA then reads all blocks
//       into shared memory (the act exchange); lane t takes one (position, super-block) pair of
//       the down rows and rows t / pairs, + slots, ...; then per output row the block partials
//       of each expert, weighted by the route weight, the reference's fixed 8-way tree
//       ((v0+v4)+(v2+v6))+((v1+v5)+(v3+v7)), + residual.
// Lane work unit: one 256-weight super-block of a row against the lane's register copy of the
// matching activation block: per 64-weight sub-block pair, dp4a over 32 B of quants and the MMVQ
// combine of vec_dot_q4_K_q8_1 / _q5_K_ (gguf.cuh:727-750, 783-813):
// dall * sum d8*(dot*sc) - dmin * sum d8*sum(q8)*m.  Integer work is the bound (the integer pipes
// issue at half the FP32 rate), so the pair index is a compile-time constant (fixed scale
// selection), the block header and fifth bits are loaded once per block, and activations are
// stored swizzled so that a quarter warp's block loads hit distinct banks.
// Every wait is bounded by a globaltimer deadline; on expiry the kernel records MMRS_ERR_TIMEOUT in
// the workspace status word, keeps every named barrier matched, drains its copies and returns.
#include <mutex>

#include "common.cuh"
#include "decode.cuh"
#include "peer.cuh"

namespace mmrs {

constexpr int kConsumerWarps = 12;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kWarps = kConsumerWarps + 1;  // + producer
constexpr int kThreads = kWarps * 32;
constexpr int kProducerWarp = kConsumerWarps;
constexpr int kMaxUnits = 80;
constexpr int kActWords = 9;  // act record words a consumer thread loads at once (384 blocks: one pass)
constexpr int kTopK = 8;
constexpr int kRouterRounds = (16 + kWarps - 1) / kWarps;
// named barriers: consumers; table ready, router partials (all threads); the eight routing
// warps' candidates written (routing warps); the slots ready (the routing warps + the producer)
constexpr int kBarConsumers = 1, kBarTable = 3, kBarRouter = 4, kBarRoute = 5, kBarCand = 6;
constexpr int kRouteWarps = 8;  // one expert a lane: E <= 256
// control words in shared memory
enum { kCtlUnits, kCtlGuUnits, kCtlGuRows, kCtlPositions, kCtlOk, kCtlFail, kCtlWords };

// Q8_1 activations in shared memory are stored swizzled: the 16-byte chunk k of a 256-value block B
// (B counted from the start of the vector, over all positions) sits at chunk slot k ^ (B & 7), so
// that the lanes of a quarter warp, each reading a whole block of a different B, hit distinct banks.
__device__ __forceinline__ int act_swz(int o) {
    return (o & ~0xff) | ((((o >> 4) & 15) ^ ((o >> 8) & 7)) << 4) | (o & 15);
}

// a: unsigned bytes, b: signed bytes.
__device__ __forceinline__ int dp4a_us(uint32_t a, int b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Scales/mins of sub-blocks 2j, 2j+1 as two packed byte pairs (get_scale_min_k4, quantized.cu:926-933).
__device__ __forceinline__ void scale_pair(const uint4 &hdr, int j, uint32_t &scp, uint32_t &mp) {
    const int sh = 16 * (j & 1);
    const uint32_t Y = hdr.y >> sh, Z = hdr.z >> sh, W = hdr.w >> sh;
    if (j < 2) {
        scp = Y & 0x3F3Fu;
        mp = Z & 0x3F3Fu;
    } else {
        scp = (W & 0x0F0Fu) | ((Y >> 2) & 0x3030u);
        mp = ((W >> 4) & 0x0F0Fu) | ((Z >> 2) & 0x3030u);
    }
}

// A lane's register copy of the activation of one 256-value block: 64 int8 x 4 as 64 ints (pair
// j: ints 16j..16j+7 the low sub-block 2j, 16j+8..16j+15 the high one) and per pair the scale
// record {d8 lo, d8 hi, d8*sum(q) lo, d8*sum(q) hi}.
struct BlockAct {
    int q[64];
    float4 ts[4];
};

// q: the block's 256 quants in the swizzled layout (B: the block's index); ts: its 4 pair records
__device__ __forceinline__ void load_block_act(const int8_t *q, int B, const float4 *ts, BlockAct &a) {
    const int4 *src = reinterpret_cast<const int4 *>(q);
#pragma unroll
    for (int k = 0; k < 16; ++k) {
        const int4 v = src[k ^ (B & 7)];
        a.q[4 * k] = v.x;
        a.q[4 * k + 1] = v.y;
        a.q[4 * k + 2] = v.z;
        a.q[4 * k + 3] = v.w;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) a.ts[j] = ts[j];
}

// One 64-weight sub-block pair J of a super-block against its activation: dp4a over the quants,
// then the MMVQ combine of vec_dot_q4_K_q8_1 / _q5_K_ (gguf.cuh:727-750, 783-813):
// dall * (d8lo*dlo*sc_lo + d8hi*dhi*sc_hi) - dmin * (d8lo*S_lo*m_lo + d8hi*S_hi*m_hi).
// J is a compile-time constant, so every shift and scale selection is fixed.
template <int TYPE, int J>
__device__ __forceinline__ float pair_dot(const uint8_t *blk, const uint4 &hdr, const uint32_t (&h)[8], const int *a,
                                          const float4 &ts) {
    int d0 = 0, d1 = 0, d2 = 0, d3 = 0;
    int b0 = 0, b1 = 0, b2 = 0, b3 = 0;
    if (TYPE == MMRS_Q5K) {
        const uint4 q0 = *reinterpret_cast<const uint4 *>(blk + 48 + 32 * J);
        const uint4 q1 = *reinterpret_cast<const uint4 *>(blk + 64 + 32 * J);
        const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
        // The fifth bits stay where they are: bit m = 2J (low sub-block) or 2J + 1 (high) of each qh
        // byte, masked, gives 2^m * hb per byte, so dp4a against the activation yields
        // 2^m * dot(hb, a), rescaled to 16 * dot(hb, a) once per pair (exact: every term carries
        // 2^m).  Likewise the high nibbles are taken in place (16 * q).  Only masks and dp4a: no
        // shifts, which issue at half rate on the same pipe as the masks.
        constexpr uint32_t ML = 0x01010101u << (2 * J), MH = 0x01010101u << (2 * J + 1);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            if (c & 1) {
                d1 = dp4a_us(w[c] & 0x0F0F0F0Fu, a[c], d1);
                d3 = dp4a_us(w[c] & 0xF0F0F0F0u, a[8 + c], d3);
                b1 = dp4a_us(h[c] & ML, a[c], b1);
                b3 = dp4a_us(h[c] & MH, a[8 + c], b3);
            } else {
                d0 = dp4a_us(w[c] & 0x0F0F0F0Fu, a[c], d0);
                d2 = dp4a_us(w[c] & 0xF0F0F0F0u, a[8 + c], d2);
                b0 = dp4a_us(h[c] & ML, a[c], b0);
                b2 = dp4a_us(h[c] & MH, a[8 + c], b2);
            }
        }
    } else {
        const uint4 q0 = *reinterpret_cast<const uint4 *>(blk + 16 + 32 * J);
        const uint4 q1 = *reinterpret_cast<const uint4 *>(blk + 32 + 32 * J);
        const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            if (c & 1) {
                d1 = dp4a_us(w[c] & 0x0F0F0F0Fu, a[c], d1);
                d3 = dp4a_us(w[c] & 0xF0F0F0F0u, a[8 + c], d3);
            } else {
                d0 = dp4a_us(w[c] & 0x0F0F0F0Fu, a[c], d0);
                d2 = dp4a_us(w[c] & 0xF0F0F0F0u, a[8 + c], d2);
            }
        }
    }
    // high nibbles were taken in place: every term carries 16 (exact shift)
    int dlo = d0 + d1, dhi = (d2 + d3) >> 4;
    if (TYPE == MMRS_Q5K) {
        const int bl = b0 + b1, bh = b2 + b3;
        dlo += J < 2 ? bl << (4 - 2 * J) : bl >> (2 * J - 4);
        dhi += J < 2 ? bh << (3 - 2 * J) : bh >> (2 * J - 3);
    }
    uint32_t scp, mp;
    scale_pair(hdr, J, scp, mp);
    // exact products: |dlo|, |dhi| < 2^17 and the 6-bit scales keep them below 2^24
    const float flo = int22_to_float(dlo) * small_uint_to_float(scp & 0xffu);
    const float fhi = int22_to_float(dhi) * small_uint_to_float(scp >> 8);
    const float sd = ts.x * flo + ts.y * fhi;
    const float sm = ts.z * small_uint_to_float(mp & 0xffu) + ts.w * small_uint_to_float(mp >> 8);
    const float2 dm = __half22float2(*reinterpret_cast<const __half2 *>(&hdr.x));
    return dm.x * sd - dm.y * sm;
}

// Dot of one 256-weight super-block (in shared memory) with its activation: pairs 0..3 in order.
template <int TYPE>
__device__ __forceinline__ float block_dot(const uint8_t *blk, const BlockAct &a) {
    const uint4 hdr = *reinterpret_cast<const uint4 *>(blk);
    uint32_t h[8];
    if (TYPE == MMRS_Q5K) {
        const uint4 h0 = *reinterpret_cast<const uint4 *>(blk + 16);
        const uint4 h1 = *reinterpret_cast<const uint4 *>(blk + 32);
        h[0] = h0.x; h[1] = h0.y; h[2] = h0.z; h[3] = h0.w;
        h[4] = h1.x; h[5] = h1.y; h[6] = h1.z; h[7] = h1.w;
    } else {
#pragma unroll
        for (int c = 0; c < 8; ++c) h[c] = 0u;
    }
    float v = pair_dot<TYPE, 0>(blk, hdr, h, a.q, a.ts[0]);
    v += pair_dot<TYPE, 1>(blk, hdr, h, a.q + 16, a.ts[1]);
    v += pair_dot<TYPE, 2>(blk, hdr, h, a.q + 32, a.ts[2]);
    v += pair_dot<TYPE, 3>(blk, hdr, h, a.q + 48, a.ts[3]);
    return v;
}

// Fixed-order sum of a row's per-block partials.
__device__ __forceinline__ float sum_blocks(const float *p, int nb) {
    float v = p[0];
#pragma unroll 4
    for (int b = 1; b < nb; ++b) v += p[b];
    return v;
}

// Distance of |y| from the nearest half-integer.  roundf(v / d) with the IEEE quotient (roundf:
// halves away from zero), |v| <= 127 d: the product v * (1/d) is within 1.5e-5 of the quotient
// (two roundings, |v/d| <= 127), so unless it lies within 1e-4 of a half-integer both round to the
// same integer; only then (or for a non-finite product, from a subnormal d) is the exact quotient
// formed, in a warp-voted branch.
__device__ __forceinline__ float half_gap(float y) {
    const float a = fabsf(y);
    return fabsf((a - floorf(a)) - 0.5f);
}

// 128 consecutive values, lane l holding values 4l..4l+3 (Q8_1 blocks of 32 over 8 lanes):
// d = amax/127, q = roundf(v/d) (quantize_q8_1, gguf.cuh:1234-1261, and quantize_silu_mul_q8_1,
// moe_gguf.cu:255-284).  Writes q (value o + i at byte act_swz(o + i) of qv), and per block the
// fp16-rounded scale d and the sum of quants S.  Out of line: it runs once per launch, and one
// copy of its code keeps the kernel's instruction footprint down.
__device__ __noinline__ void quant128(float4 v, int8_t *qv, int o, float *d, int *S, int lane) {
    float amax = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
#pragma unroll
    for (int m = 4; m > 0; m >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, m));
    const float dd = __fdiv_rn(amax, 127.0f);
    int q0 = 0, q1 = 0, q2 = 0, q3 = 0;
    bool exact = false;
    float y0 = 0.f, y1 = 0.f, y2 = 0.f, y3 = 0.f;
    if (amax != 0.f) {
        const float inv = __frcp_rn(dd);
        y0 = v.x * inv;
        y1 = v.y * inv;
        y2 = v.z * inv;
        y3 = v.w * inv;
        q0 = (int)roundf(y0);
        q1 = (int)roundf(y1);
        q2 = (int)roundf(y2);
        q3 = (int)roundf(y3);
        exact = !(half_gap(y0) > 1e-4f) || !(half_gap(y1) > 1e-4f) || !(half_gap(y2) > 1e-4f) ||
                !(half_gap(y3) > 1e-4f);
    }
    if (__any_sync(0xffffffffu, exact) && exact) {
        if (!(half_gap(y0) > 1e-4f)) q0 = (int)roundf(__fdiv_rn(v.x, dd));
        if (!(half_gap(y1) > 1e-4f)) q1 = (int)roundf(__fdiv_rn(v.y, dd));
        if (!(half_gap(y2) > 1e-4f)) q2 = (int)roundf(__fdiv_rn(v.z, dd));
        if (!(half_gap(y3) > 1e-4f)) q3 = (int)roundf(__fdiv_rn(v.w, dd));
    }
    *reinterpret_cast<int *>(qv + act_swz(o + 4 * lane)) =
        (q0 & 0xff) | ((q1 & 0xff) << 8) | ((q2 & 0xff) << 16) | ((q3 & 0xff) << 24);
    int s = q0 + q1 + q2 + q3;
#pragma unroll
    for (int m = 4; m > 0; m >>= 1) s += __shfl_xor_sync(0xffffffffu, s, m);
    if ((lane & 7) == 0) {
        d[lane >> 3] = __half2float(__float2half_rn(dd));
        S[lane >> 3] = s;
    }
}

// One Q8_1 block of 32 values, lane l holding value l: the quant128 arithmetic (d = amax/127,
// q = roundf(v/d), fp16-rounded d, sum of quants), published as the block's nine tagged words:
// quants 4j..4j+3 (word j < 8) and {fp16 bits of d, int16 sum of quants} (word 8), each with the
// launch tag in its upper half (relaxed 64-bit stores: no fence).
__device__ __forceinline__ void publish_block(float v, unsigned long long *rec, uint32_t tag, int lane) {
    const float amax = warp_max_butterfly(fabsf(v));
    const float dd = __fdiv_rn(amax, 127.0f);
    int qi = 0;
    bool exact = false;
    if (amax != 0.f) {
        const float y = v * __frcp_rn(dd);
        qi = (int)roundf(y);
        exact = !(half_gap(y) > 1e-4f);
    }
    if (__any_sync(0xffffffffu, exact) && exact) qi = (int)roundf(__fdiv_rn(v, dd));
    int sq = qi;
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, m);
    const uint32_t qb = (uint32_t)qi & 0xffu;
    uint32_t w = qb;
    w |= __shfl_down_sync(0xffffffffu, qb, 1) << 8;
    w |= __shfl_down_sync(0xffffffffu, qb, 2) << 16;
    w |= __shfl_down_sync(0xffffffffu, qb, 3) << 24;
    const unsigned long long hi = (unsigned long long)tag << 32;
    if ((lane & 3) == 0) st_relaxed_gpu_u64(rec + (lane >> 2), hi | w);
    if (lane == 0) {
        const uint32_t dbits = __half_as_ushort(__float2half_rn(dd));  // |sum of quants| <= 32 * 127
        st_relaxed_gpu_u64(rec + 8, hi | dbits | ((uint32_t)(sq & 0xffff) << 16));
    }
}

// The CTA's gate/up range of (position, row) pairs: whole Q8_1 blocks of 32 rows, so that every
// block of act is quantised by the one CTA that computed it.
__device__ __forceinline__ void gu_range(int cta, int G, int nvs, int I, int &p0, int &p1) {
    const uint32_t nblk = (uint32_t)(nvs * I / 32);  // cta * nblk < 2^31: G <= 256, 8 I / 32 <= 1536
    p0 = 32 * (int)((uint32_t)cta * nblk / (uint32_t)G);
    p1 = 32 * (int)((uint32_t)(cta + 1) * nblk / (uint32_t)G);
}

// Per-task scale records from per-block (d, S) arrays: nt tasks, 2 blocks each.
__device__ __forceinline__ void build_task_scales(float4 *ts, const float *d, const int *S, int nt, int tid, int nthr) {
    for (int t = tid; t < nt; t += nthr) {
        const float dl = d[2 * t], dh = d[2 * t + 1];
        ts[t] = make_float4(dl, dh, dl * (float)S[2 * t], dh * (float)S[2 * t + 1]);
    }
}

// Bounded wait until unit k has landed in stage st: first the stage's ticket (the producer has
// issued unit k there; a lane may reach unit k before unit k - stages has been freed), then the
// phase of the stage's full barrier.
__device__ __forceinline__ bool wait_unit(uint64_t *full, const int *ticket, int k, int st, int stages,
                                          uint64_t deadline) {
    uint32_t spins = 0;
    while (*reinterpret_cast<const volatile int *>(&ticket[st]) != k) {
        if ((++spins & 1023u) == 0 && globaltimer_ns() > deadline) return false;
    }
    return mbar_wait_sleep(&full[st], (uint32_t)(k / stages) & 1u, deadline);
}

// One thread's bounded wait until an exchange counter reaches `target` (wrap-safe).  None of the
// decode kernel's polls sleep between reads (__nanosleep): on B200 a warp woken from a 32-128 ns
// sleep was measured to resume microseconds later, which put whole microseconds on the routing
// and exchange paths; a spin issues one load per memory round trip.
__device__ __forceinline__ bool wait_count(const uint32_t *cnt, uint32_t target, uint64_t deadline) {
    uint32_t spins = 0;
    while ((int)(ld_relaxed_gpu(cnt) - target) < 0) {  // one L2 round trip a poll
        if ((++spins & 63u) == 0 && globaltimer_ns() > deadline) return false;
    }
    return true;
}

// arrive.expect_tx whose arrival state is not returned (the issuing thread does not wait for it)
__device__ __forceinline__ void mbar_arrive_expect_tx_sink(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

// Shared-memory add with acquire-release semantics at CTA scope (returns the old value): the
// warps that finished a copy unit before release their reads of its stage to the last finisher.
__device__ __forceinline__ int atom_add_acq_rel_cta(int *p, int v) {
    int old;
    asm volatile("atom.acq_rel.cta.shared::cta.add.u32 %0, [%1], %2;" : "=r"(old) : "r"(smem_u32(p)), "r"(v) : "memory");
    return old;
}

// Order-preserving selection key of sigmoid(l) + bias (-0 ranks as +0).
__device__ __forceinline__ uint32_t sel_key(float sg, float b) {
    float sv = sg + b;
    if (sv == 0.0f) sv = 0.0f;
    const uint32_t u = __float_as_uint(sv);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Copy unit: .x kind (0 gate, 1 up, 2 down), .y slot position, .z first row, .w rows.
// Sub-unit: .x unit, .y first row within the unit | rows << 16.
// Floats of the per-block partial buffer: the gate/up rows' and, after them, the down rows'.
__host__ __device__ inline size_t decode_part_floats(const DecodeParams &p) {
    const size_t gu = (size_t)2 * p.act_slots * ((p.H / QK_K) | 1), dn = (size_t)kTopK * p.res_slots * (p.I / QK_K);
    return gu > dn ? gu : dn;
}

struct DecodeSmem {
    uint8_t *stages;
    uint64_t *full;
    int8_t *xq;                // [H]
    float *xd;                 // [H/32]
    int *xS;                   // [H/32]
    float4 *xts;               // [H/64]
    int8_t *aq_s;              // [8][I] (positions)
    float *ad_s;               // [8][I/32]
    int *aS_s;                 // [8][I/32]
    float4 *ats;               // [8][I/64]
    float *part;               // router slice sums [2][8]
    uint2 *cand;               // [64] routing candidates {key, expert id}, warp w's at 8 w + rank
    float *csig;               // [64] their sigmoids
    float *slotsig;            // [8] sigmoid of the expert of each slot
    int *ids;                  // [8] expert of each slot (-1: none, or another rank's)
    int *vslot;                // [8] slot of each position (the computed slots in order)
    int *posof;                // [8] position of each slot (-1: not computed here)
    float *w;                  // [8]
    float *dn_acc;             // [res_slots][8] weighted expert rows of this CTA's output range
    float *bpart;              // per-block partial sums: gate/up [2][act_slots][H/256 | 1], then
                               // down [positions][res_slots][I/256]
    float *res_s;              // [res_slots]
    int4 *units;               // [kMaxUnits]
    int *unit_off;             // [kMaxUnits] first row of a gate/up unit in the CTA's range
    const uint8_t **usrc;      // [kMaxUnits] global source of the unit's copy
    uint32_t *ubytes;          // [kMaxUnits] its size
    int2 *rowmap;              // [2 act_slots] gate/up row g: {unit | row in unit << 16, partial row}
    int *ticket;               // [stages] unit last issued into each stage
    int *done;                 // [stages] super-blocks of the stage's unit finished
    int *ctl;                  // [kCtlWords]
};

// Copy-table structure of a CTA for nv computed positions (one producer lane each): lane c
// describes gate/up chunk c of the CTA's (position, row) range (its position, first row, rows,
// offset in the range); units 2c / 2c + 1 are the chunk's gate / up rows, then one down unit per
// position (all of the CTA's output rows); the row map gives each gate/up row its unit, its row
// in the unit and its partial-sum row (gate rows first, then up rows).  It depends on the number
// of positions only, not on the experts (the source addresses are filled in once the routing is
// known).  Out of line: one copy of its code for both call sites.
struct TableLane {
    int pos, row0, n, off, n_chunks, cnt;
};
__device__ __noinline__ TableLane table_structure(int cta, int G, int nv, int I, int U_gu, int lane, uint32_t gu_row_bytes,
                                                  uint32_t dn_row_bytes, int nres, int dn_r0, int4 *units, int *unit_off,
                                                  uint32_t *ubytes, int2 *rowmap) {
    TableLane t = {-1, 0, 0, 0, 0, 0};
    int gu_p0, gu_p1;
    gu_range(cta, G, nv, I, gu_p0, gu_p1);
    int c_left = lane;
    for (int pos = gu_p0 / I, q = gu_p0; q < gu_p1; ++pos) {
        const int seg_end = min(gu_p1, (pos + 1) * I);
        const int nc = (seg_end - q + U_gu - 1) / U_gu;
        if (c_left >= 0 && c_left < nc) {
            const int r = q + c_left * U_gu;
            t.pos = pos;
            t.row0 = r - pos * I;
            t.n = min(U_gu, seg_end - r);
            t.off = r - gu_p0;
        }
        c_left -= nc;
        t.n_chunks += nc;
        q = seg_end;
    }
    t.cnt = gu_p1 - gu_p0;
    if (t.pos >= 0) {
        for (int h = 0; h < 2; ++h) {
            const int k = 2 * lane + h;
            units[k] = make_int4(h, t.pos, t.row0, t.n);
            unit_off[k] = t.off;
            ubytes[k] = gu_row_bytes * (uint32_t)t.n;
#pragma unroll 1
            for (int r = 0; r < t.n; ++r) rowmap[2 * t.off + h * t.n + r] = make_int2(k | (r << 16), h * t.cnt + t.off + r);
        }
    }
    if (nres > 0 && lane < nv) {
        const int k = 2 * t.n_chunks + lane;
        units[k] = make_int4(2, lane, dn_r0, nres);
        unit_off[k] = 0;
        ubytes[k] = dn_row_bytes * (uint32_t)nres;
    }
    return t;
}

// GU / DN: GGUF types of the gate/up and down matrices (one instantiation per pair keeps each
// launched kernel's code to the dot products it runs).
template <int GU, int DN>
__global__ void __launch_bounds__(kThreads, 1) moe_decode_fused_kernel(const __grid_constant__ DecodeParams p) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, cta = blockIdx.x;
    const int H = p.H, I = p.I, E = p.E;
    const uint64_t t_start = globaltimer_ns();
    const uint64_t deadline = t_start + p.timeout_ns;
    // the CTA's output rows (cta * H < 2^31: G <= 256, H <= 4096)
    const int dn_r0 = (int)((uint32_t)(cta * H) / (uint32_t)G), dn_r1 = (int)((uint32_t)((cta + 1) * H) / (uint32_t)G);
    const int nres = dn_r1 - dn_r0;

    // ---- P0 loads first: the CTA's router rows (weights: they do not depend on the previous
    // kernel in the stream, so they are requested before the programmatic-launch wait), then,
    // after it, the matching x slices ---------------------------------------------------------
    const int slice = H / 8, groups = slice / 4;
    float4 xx[kRouterRounds][4], wv[kRouterRounds][4];
#pragma unroll
    for (int r = 0; r < kRouterRounds; ++r) {
        const int pi = warp + kWarps * r, sl = pi & 7, le = pi >> 3;
        const int e = cta + G * le;
        if (pi < 16 && p.internal_routing && e < E) {
            const float4 *wr = reinterpret_cast<const float4 *>(p.router + (size_t)e * H + sl * slice);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int g = lane + 32 * i;
                if (g < groups) wv[r][i] = __ldg(wr + g);
            }
        }
    }
    // the routing lane's selection bias (a weight as well)
    const int route_e = 32 * warp + lane;
    const float route_bias = (p.internal_routing && warp < kRouteWarps && route_e < E) ? __ldg(p.bias + route_e) : 0.f;
    // everything below reads the previous kernel's outputs (x, the workspace)
    asm volatile("griddepcontrol.wait;" ::: "memory");
#pragma unroll
    for (int r = 0; r < kRouterRounds; ++r) {
        const int pi = warp + kWarps * r, sl = pi & 7, le = pi >> 3;
        const int e = cta + G * le;
        if (pi < 16 && p.internal_routing && e < E) {
            const float4 *xs = reinterpret_cast<const float4 *>(p.x + sl * slice);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int g = lane + 32 * i;
                if (g < groups) {
                    xx[r][i] = __ldg(xs + g);
                }
            }
        }
    }
    // this launch's tag: one more than this CTA's last (its own arrival word counts its launches)
    const uint32_t tag = __ldcg(&p.ctl->arrive[cta]) + 1u;
    if (tid == 0 && p.trace) p.trace[cta * kTraceSlots + 0] = t_start;

    DecodeSmem s;
    {
        uint8_t *ptr = smem_raw;
        auto take = [&](size_t bytes) {
            uint8_t *r = ptr;
            ptr += (bytes + 15) / 16 * 16;
            return r;
        };
        s.stages = take((size_t)p.stages * p.stage_bytes);
        s.full = reinterpret_cast<uint64_t *>(take(sizeof(uint64_t) * p.stages));
        s.xq = reinterpret_cast<int8_t *>(take(H));
        s.xd = reinterpret_cast<float *>(take(sizeof(float) * (H / 32)));
        s.xS = reinterpret_cast<int *>(take(sizeof(int) * (H / 32)));
        s.xts = reinterpret_cast<float4 *>(take(sizeof(float4) * (H / 64)));
        s.aq_s = reinterpret_cast<int8_t *>(take((size_t)kTopK * I));
        s.ad_s = reinterpret_cast<float *>(take(sizeof(float) * kTopK * (I / 32)));
        s.aS_s = reinterpret_cast<int *>(take(sizeof(int) * kTopK * (I / 32)));
        s.ats = reinterpret_cast<float4 *>(take(sizeof(float4) * kTopK * (I / 64)));
        s.part = reinterpret_cast<float *>(take(sizeof(float) * 16));
        s.cand = reinterpret_cast<uint2 *>(take(sizeof(uint2) * 64));
        s.csig = reinterpret_cast<float *>(take(sizeof(float) * 64));
        s.slotsig = reinterpret_cast<float *>(take(sizeof(float) * kTopK));
        s.ids = reinterpret_cast<int *>(take(sizeof(int) * kTopK));
        s.vslot = reinterpret_cast<int *>(take(sizeof(int) * kTopK));
        s.posof = reinterpret_cast<int *>(take(sizeof(int) * kTopK));
        s.w = reinterpret_cast<float *>(take(sizeof(float) * kTopK));
        s.dn_acc = reinterpret_cast<float *>(take(sizeof(float) * kTopK * p.res_slots));
        s.bpart = reinterpret_cast<float *>(take(sizeof(float) * decode_part_floats(p)));
        s.res_s = reinterpret_cast<float *>(take(sizeof(float) * p.res_slots));
        s.units = reinterpret_cast<int4 *>(take(sizeof(int4) * kMaxUnits));
        s.unit_off = reinterpret_cast<int *>(take(sizeof(int) * kMaxUnits));
        s.usrc = reinterpret_cast<const uint8_t **>(take(sizeof(void *) * kMaxUnits));
        s.ubytes = reinterpret_cast<uint32_t *>(take(sizeof(uint32_t) * kMaxUnits));
        s.rowmap = reinterpret_cast<int2 *>(take(sizeof(int2) * 2 * p.act_slots));
        s.ticket = reinterpret_cast<int *>(take(sizeof(int) * p.stages));
        s.done = reinterpret_cast<int *>(take(sizeof(int) * p.stages));
        s.ctl = reinterpret_cast<int *>(take(sizeof(int) * kCtlWords));
        // the carve-up must fit the dynamic allocation computed by decode_smem_bytes()
        uint32_t dyn = 0;
        asm volatile("mov.u32 %0, %%dynamic_smem_size;" : "=r"(dyn));
        if ((size_t)(ptr - smem_raw) > dyn) {
            if (tid == 0) atomicExch(&p.ctl->status, (uint32_t)MMRS_ERR_LAUNCH);
            return;
        }
    }
    if (tid == 0) {
        for (int i = 0; i < p.stages; ++i) {
            mbar_init(&s.full[i], 1);
            s.ticket[i] = -1;
            s.done[i] = 0;
        }
        fence_mbar_init();
        for (int i = 0; i < kCtlWords; ++i) s.ctl[i] = 0;
        s.ctl[kCtlOk] = 1;  // cleared by a routing lane whose score wait expires
        if (cta == 0) p.ctl->zero_bytes = p.zero_bytes;
    }

    // ---- P0: router slices -------------------------------------------------------------------
#pragma unroll
    for (int r = 0; r < kRouterRounds; ++r) {
        const int pi = warp + kWarps * r, sl = pi & 7, le = pi >> 3;
        if (!(pi < 16 && p.internal_routing && cta + G * le < E)) continue;
        float acc = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int g = lane + 32 * i;
            if (g < groups) {
                acc = fmaf(wv[r][i].x, xx[r][i].x, acc);
                acc = fmaf(wv[r][i].y, xx[r][i].y, acc);
                acc = fmaf(wv[r][i].z, xx[r][i].z, acc);
                acc = fmaf(wv[r][i].w, xx[r][i].w, acc);
            }
        }
        acc = warp_sum_butterfly(acc);
        if (lane == 0) s.part[le * 8 + sl] = acc;
    }
    named_sync(kBarRouter, kThreads);
    if (p.internal_routing && tid < 2 * kScoreReplicas) {
        // thread t publishes the score of the CTA's expert t / kScoreReplicas into copy
        // t % kScoreReplicas (the 16 threads of an expert form the same value)
        const int le = tid / kScoreReplicas, ee = cta + G * le;
        if (ee < E) {
            const float *q = s.part + le * 8;
            const float lg = ((q[0] + q[1]) + (q[2] + q[3])) + ((q[4] + q[5]) + (q[6] + q[7]));
            // the sigmoid (minimax_moe_decode_topk's arithmetic), published with this launch's tag
            // in the same 64-bit word
            const float sg = __fdiv_rn(1.0f, 1.0f + expf(-lg));
            publish_gpu_u64(p.score + (size_t)(tid % kScoreReplicas) * 256 + ee,
                            ((unsigned long long)tag << 32) | __float_as_uint(sg));
        }
    }
    if (tid == 0 && p.trace) p.trace[cta * kTraceSlots + 1] = globaltimer_ns();

    const size_t gu_row_bytes = kq_row_bytes(p.gu_type, H);
    const size_t dn_row_bytes = kq_row_bytes(p.dn_type, I);
    const size_t gu_expert_bytes = gu_row_bytes * I;
    const size_t dn_expert_bytes = dn_row_bytes * H;
    const int U_gu = p.gu_unit_rows;
    const int NBg = H / QK_K, NBd = I / QK_K;  // super-blocks of a gate/up row, of a down row
    const int NBgs = NBg | 1;  // row stride of the gate/up block partials (odd: conflict-free row sums)

    // Issue copy unit k into ring stage k % stages (one thread).  The first `stages` units are
    // issued by the producer warp once the table is built; every later unit by the consumer lane
    // that completes the last super-block of unit k - stages, which frees that stage.
    auto issue = [&](int k) {
        const int st = k % p.stages;
        *reinterpret_cast<volatile int *>(&s.ticket[st]) = k;
        const uint32_t bytes = s.ubytes[k];
        if (p.trace) {
            if (k == 0) p.trace[cta * kTraceSlots + 8] = globaltimer_ns();
            if (k == s.ctl[kCtlGuUnits]) p.trace[cta * kTraceSlots + 10] = globaltimer_ns();
            if (k == s.ctl[kCtlUnits] - 1) p.trace[cta * kTraceSlots + 9] = globaltimer_ns();
        }
        mbar_arrive_expect_tx_sink(&s.full[st], bytes);
        // the expert weights are read once per token: first out of L2, so the stream does not
        // push the lines the CTAs exchange out of it (measured ~1 % faster)
        uint64_t pol;
        asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
        asm volatile(
            "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
                smem_u32(s.stages + (size_t)st * p.stage_bytes)),
            "l"(s.usrc[k]), "r"(bytes), "r"(smem_u32(&s.full[st])), "l"(pol)
            : "memory");
    };

    if (warp == kProducerWarp) {
        // ================================ producer warp ===================================
        // The copy-table structure (table_structure) is built while the routing warps wait for
        // the scores when the number of computed positions is known in advance.
        TableLane tl;
        auto structure = [&](int nv) {
            tl = table_structure(cta, G, nv, I, U_gu, lane, (uint32_t)gu_row_bytes, (uint32_t)dn_row_bytes, nres, dn_r0,
                                 s.units, s.unit_off, s.ubytes, s.rowmap);
        };
        // every slot is computed here unless experts are split over ranks
        const bool compact = p.world > 1 && p.ep;
        const int nv_guess = compact ? -1 : kTopK;
        if (nv_guess > 0) structure(nv_guess);
        // the routing warps wait for the scores; their candidates (and verdict) arrive here
        named_sync(kBarCand, 32 * (kRouteWarps + 1));
        const bool ok = s.ctl[kCtlOk] != 0;
        if (lane == 0 && p.trace) p.trace[cta * kTraceSlots + 2] = globaltimer_ns();
        // ---- slots (merged by the routing warps) and their weights ---------------------------------
        int slot_id = -1;  // lane k < 8: expert of slot k
        float slot_w = 0.f;
        if (p.internal_routing) {
            if (ok) {
                // the routing warps wrote the expert and sigmoid of each slot
                if (lane < kTopK) slot_id = s.ids[lane];
                // weights: sig / ((v0+v4)+(v2+v6))+((v1+v5)+(v3+v7)), lane k keeps w_k
                const float my_sig = lane < kTopK ? s.slotsig[lane] : 0.f;
                float v[kTopK];
#pragma unroll
                for (int k = 0; k < kTopK; ++k) v[k] = __shfl_sync(0xffffffffu, my_sig, k);
                const float denom = ((v[0] + v[4]) + (v[2] + v[6])) + ((v[1] + v[5]) + (v[3] + v[7]));
                if (lane < kTopK) {
                    slot_w = __fdiv_rn(my_sig, denom);
                    if (cta == 0) {
                        if (p.topk_ids_out) p.topk_ids_out[lane] = (uint32_t)slot_id;
                        if (p.topk_w_out) p.topk_w_out[lane] = slot_w;
                    }
                }
            }
        } else {
            // caller-supplied (route, expert) pairs in expert order, weights by route; routes
            // outside [0, 8) and invalid experts contribute nothing (moe_gguf.cu:311)
            if (lane < kTopK) {
                s.ids[lane] = -1;
                s.w[lane] = 0.f;
            }
            __syncwarp();
            if (ok && lane < kTopK) {
                const int route = p.ext_route[lane];
                const int e = p.ext_expert[lane];
                if (route >= 0 && route < kTopK) {
                    s.ids[route] = (e >= 0 && e < E) ? e : -1;
                    s.w[route] = p.ext_w[route];
                }
            }
            __syncwarp();
            if (lane < kTopK) {
                slot_id = s.ids[lane];
                slot_w = s.w[lane];
            }
            __syncwarp();
        }
        if (lane == 0 && p.trace) p.trace[cta * kTraceSlots + 14] = globaltimer_ns();
        // ---- positions: the computed slots in order (expert parallel: this rank's only) ------
        int id = (ok && lane < kTopK) ? slot_id : -1;
        if (compact && id >= 0 && id % p.world != p.rank) id = -1;
        const bool keep = lane < kTopK && id >= 0;
        const uint32_t kept = __ballot_sync(0xffffffffu, keep);
        const int nvs = __popc(kept);
        if (lane < kTopK) {
            s.ids[lane] = id;
            s.w[lane] = slot_w;
            s.posof[lane] = keep ? __popc(kept & ((1u << lane) - 1u)) : -1;
            if (keep) s.vslot[__popc(kept & ((1u << lane) - 1u))] = lane;
        }
        if (nvs != nv_guess) structure(nvs);
        __syncwarp();
        // ---- source addresses of the units, then the first ring fill (one unit per lane);
        // later units are issued by the consumer lanes ------------------------------------------
        const int n_gu_units = 2 * tl.n_chunks;
        const int n_dn_units = nres > 0 ? nvs : 0;
        if (tl.pos >= 0) {
            const size_t e = (size_t)s.ids[s.vslot[tl.pos]];
            s.usrc[2 * lane] = p.gate + e * gu_expert_bytes + (size_t)tl.row0 * gu_row_bytes;
            s.usrc[2 * lane + 1] = p.up + e * gu_expert_bytes + (size_t)tl.row0 * gu_row_bytes;
        }
        if (lane < n_dn_units) {
            const size_t e = (size_t)s.ids[s.vslot[lane]];
            s.usrc[n_gu_units + lane] = p.down + e * dn_expert_bytes + (size_t)dn_r0 * dn_row_bytes;
        }
        if (lane == 0) {
            s.ctl[kCtlUnits] = n_gu_units + n_dn_units;
            s.ctl[kCtlGuUnits] = n_gu_units;
            s.ctl[kCtlGuRows] = 2 * tl.cnt;
            s.ctl[kCtlPositions] = nvs;
            s.ctl[kCtlOk] = ok ? 1 : 0;
        }
        __syncwarp();
        if (lane == 0 && p.trace) p.trace[cta * kTraceSlots + 15] = globaltimer_ns();
        if (ok && lane < min(n_gu_units + n_dn_units, p.stages)) issue(lane);
        if (lane == 0 && p.trace) p.trace[cta * kTraceSlots + 3] = globaltimer_ns();
        __syncwarp();
        named_arrive(kBarTable, kThreads);  // table complete: the consumers may start
        __syncwarp();
        return;
    }

    // ================================ consumer warps ======================================
    // Routing warps first: the copy table waits for their candidates.  Routing warp w computed
    // the router slice w of the CTA's first expert, so it holds x's slice w in registers (lane l:
    // values 4l..4l+3 of each 128-value chunk), which it quantises (Q8_1) once its candidates
    // are out, while the producer merges them.  Without that slice (external
    // routing, a CTA without a first expert, H not a multiple of 1024) the other consumer warps
    // load and quantise x.  They load the residual.
    const bool xq_router = p.internal_routing && H % 1024 == 0 && cta < E;
    if (warp < kRouteWarps) {
        // this launch's score of expert e (bounded wait for its tag), the selection key, this
        // warp's top-8 of its 32 experts by rank, then the global top-8 of the 64 candidates
        const int e = route_e;
        // each routing lane polls its expert's tagged score in the CTA's copy directly (one
        // coalesced 256-byte request per warp and round: ~10 requests per L2 line and round over
        // the grid)
        if (p.internal_routing) {
            uint32_t key = 0u;  // experts >= E are never selected (E >= 8 real keys are > 0)
            float sg = 0.f;
            if (e < E) {
                const unsigned long long *word = p.score + (size_t)(cta % kScoreReplicas) * 256 + e;
                unsigned long long v = ld_relaxed_gpu_u64(word);
                uint32_t spins = 0;
                while ((uint32_t)(v >> 32) != tag) {  // one L2 round trip a poll
                    if ((++spins & 63u) == 0 && globaltimer_ns() > deadline) {
                        atomicExch(&p.ctl->status, (uint32_t)MMRS_ERR_TIMEOUT);
                        s.ctl[kCtlOk] = 0;
                        break;
                    }
                    v = ld_relaxed_gpu_u64(word);
                }
                if (tid == 0 && p.trace) p.trace[cta * kTraceSlots + 19] = globaltimer_ns();
                sg = __uint_as_float((uint32_t)v);
                key = sel_key(sg, route_bias);
            }
            // rank of this lane's expert among the warp's 32: lanes with a larger key, or an equal
            // key and a lower expert id (the stable descending order); the warp's best 8 go to
            // shared memory in rank order
            int rank = 0;
#pragma unroll 8
            for (int j = 0; j < 32; ++j) {
                const uint32_t kj = __shfl_sync(0xffffffffu, key, j);
                rank += (int)(kj > key) | ((int)(kj == key) & (int)(j < lane));
            }
            if (rank < kTopK) {
                s.cand[8 * warp + rank] = make_uint2(key, (uint32_t)e);
                s.csig[8 * warp + rank] = sg;
            }
            if (tid == 0 && p.trace) p.trace[cta * kTraceSlots + 13] = globaltimer_ns();
            if (lane == 0 && p.trace) p.trace[cta * kTraceSlots + 24 + warp] = globaltimer_ns();
            named_sync(kBarRoute, 32 * kRouteWarps);
            // The global top-8 from the 64 candidates (every warp's list holds its share of it):
            // candidate 8 w + (lane & 7)'s rank among all 64 in the same order, lanes l, l ^ 8,
            // l ^ 16, l ^ 24 counting over 16 candidates each; ranks below 8 are the slots.
            const int ci = 8 * warp + (lane & 7);
            const uint2 me = s.cand[ci];
            const uint4 *grp = reinterpret_cast<const uint4 *>(s.cand + 16 * (lane >> 3));
            int gr = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) {  // branch-free: (key greater) | (key equal & id lower)
                const uint4 q = grp[j];
                gr += (int)(q.x > me.x) | ((int)(q.x == me.x) & (int)(q.y < me.y));
                gr += (int)(q.z > me.x) | ((int)(q.z == me.x) & (int)(q.w < me.y));
            }
            gr += __shfl_xor_sync(0xffffffffu, gr, 8);
            gr += __shfl_xor_sync(0xffffffffu, gr, 16);
            if (lane < 8 && gr < kTopK) {
                s.ids[gr] = (int)me.y;
                s.slotsig[gr] = s.csig[ci];
            }
            if (tid == 0 && p.trace) p.trace[cta * kTraceSlots + 20] = globaltimer_ns();
        }
        named_arrive(kBarCand, 32 * (kRouteWarps + 1));
        if (xq_router) {
            const int cps = slice / 128;  // chunks per router slice
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int c = warp * cps + i;
                if (i < cps) quant128(xx[0][i], s.xq, c * 128, s.xd + c * 4, s.xS + c * 4, lane);
            }
        }
    } else {
        const int nxc = H / 128, xw = warp - kRouteWarps, xt = tid - 32 * kRouteWarps;
        constexpr int kXWarps = kConsumerWarps - kRouteWarps;
        for (int c = xw; c < nxc && !xq_router; c += kXWarps) {
            const float4 xv = __ldg(reinterpret_cast<const float4 *>(p.x) + c * 32 + lane);
            quant128(xv, s.xq, c * 128, s.xd + c * 4, s.xS + c * 4, lane);
        }
        for (int r = xt; r < nres; r += 32 * kXWarps) s.res_s[r] = p.residual ? __ldg(p.residual + dn_r0 + r) : 0.f;
    }
    named_sync(kBarConsumers, kConsumerThreads);  // x's Q8_1 blocks are complete
    build_task_scales(s.xts, s.xd, s.xS, H / 64, tid, kConsumerThreads);
    named_sync(kBarConsumers, kConsumerThreads);  // and their scale records
    if (tid == 0 && p.trace) p.trace[cta * kTraceSlots + 12] = globaltimer_ns();
    // Gate/up lanes: lane t holds the activation of x block t % NBg and computes that block of
    // rows t / NBg, t / NBg + slots, ... of the CTA's gate/up rows (in unit order).
    const int g_slots = kConsumerThreads / NBg;
    const bool g_lane = tid < NBg * g_slots;
    const int g_sb = tid % NBg, g_first = tid / NBg;
    BlockAct act;
    load_block_act(s.xq + QK_K * g_sb, g_sb, s.xts + 4 * g_sb, act);
    named_sync(kBarTable, kThreads);
    const bool ok1 = s.ctl[kCtlOk] != 0;
    const int nvs = s.ctl[kCtlPositions], n_units = s.ctl[kCtlUnits], n_gu_units = s.ctl[kCtlGuUnits];
    const int n_gu_rows = s.ctl[kCtlGuRows], cnt = n_gu_rows / 2;
    bool aborted = !ok1;
    // Gate/up: the lanes of a warp finished one super-block each (valid) of units k: per unit, the
    // lowest such lane adds the group's count to the stage's counter (its acquire-release covers
    // the group's reads of the stage, ordered before it by the warp sync); the lane that completes
    // the unit's rows x blocks frees the stage and issues unit k + stages into it.  The warp sync
    // is safe only while one warp's rows of a round (at most 31 / NBg + 2 consecutive rows, in as
    // many units) fit in the ring: a lane must never wait for a unit that its own warp keeps
    // unfreed.  Otherwise (small H) every lane counts its own block.
    const bool lane_counts = 31 / NBg + 2 > p.stages;
    auto finish = [&](bool valid, int k, int st, int total) {
        bool leader = valid;
        int n = 1;
        if (!lane_counts) {
            __syncwarp();
            const unsigned grp = __match_any_sync(0xffffffffu, valid ? k : -1);
            leader = valid && lane == __ffs(grp) - 1;
            n = __popc(grp);
        }
        if (leader) {
            const int old = atom_add_acq_rel_cta(&s.done[st], n);
            if (old + n == total) {
                s.done[st] = 0;
                if (k + p.stages < n_units && !aborted) issue(k + p.stages);
            }
        }
    };
    auto wait_landed = [&](int k, int st) {
        if (!aborted && !wait_unit(s.full, s.ticket, k, st, p.stages, deadline)) {
            atomicExch(&p.ctl->status, (uint32_t)MMRS_ERR_TIMEOUT);
            s.ctl[kCtlFail] = 1;  // the CTA drains its ring before it retires
            aborted = true;
        }
    };

    // ---- P2: gate / up: one super-block per lane and round -----------------------------------
    {
        constexpr int BB = GU == MMRS_Q5K ? Q5K_BYTES : Q4K_BYTES;
        const int rounds = (n_gu_rows + g_slots - 1) / g_slots;
        for (int m = 0; m < rounds; ++m) {
            const int g = g_first + m * g_slots;
            const bool valid = g_lane && g < n_gu_rows;
            int k = -1, st = 0, total = 0;
            if (valid) {
                const int2 rm = s.rowmap[g];
                k = rm.x & 0xffff;
                st = k % p.stages;
                total = s.units[k].w * NBg;
                wait_landed(k, st);
                float v = 0.f;
                if (!aborted)
                    v = block_dot<GU>(s.stages + (size_t)st * p.stage_bytes + (size_t)(rm.x >> 16) * gu_row_bytes + BB * g_sb, act);
                s.bpart[rm.y * NBgs + g_sb] = v;
            }
            finish(valid, k, st, total);
        }
        __syncwarp();  // a leader lane may still be issuing: the warp meets the barrier converged
    }

    // ---- P3: Q8_1 of act for the CTA's blocks, grid barrier #2, copy of the whole vector ---------
    named_sync(kBarConsumers, kConsumerThreads);  // every gate/up block of this CTA is done
    if (tid == 0 && p.trace) p.trace[cta * kTraceSlots + 4] = globaltimer_ns();
    {
        int gu_p0, gu_p1;
        gu_range(cta, G, nvs, I, gu_p0, gu_p1);
        // one warp per block of 32 rows: lane l sums the block partials of gate row 32 b + l
        // (partial row i) and of its up row (partial row cnt + i), forms act = up * silu(gate)
        // (moe_gguf.cu:272-273), and the warp quantises the block (quantize_silu_mul_q8_1,
        // moe_gguf.cu:255-284) and publishes it
        for (int b = gu_p0 / 32 + warp; b < gu_p1 / 32 && !aborted; b += kConsumerWarps) {
            const int i = 32 * b - gu_p0 + lane;
            if (tid == 0 && p.trace) p.trace[cta * kTraceSlots + 21] = globaltimer_ns();
            const float gv = sum_blocks(s.bpart + i * NBgs, NBg);
            const float uv = sum_blocks(s.bpart + (cnt + i) * NBgs, NBg);
            const float av = uv * __fdiv_rn(gv, 1.0f + expf(-gv));
            if (tid == 0 && p.trace) p.trace[cta * kTraceSlots + 23] = globaltimer_ns();
            publish_block(av, p.arec + (size_t)9 * b, tag, lane);
        }
        if (tid == 0 && p.trace) p.trace[cta * kTraceSlots + 22] = globaltimer_ns();
    }
    // ---- the act exchange (in place of a grid barrier): this CTA's records are written, so it
    // counts itself in; one thread waits until every CTA has, then the consumer threads read the
    // record words coalesced (thread t: words t, t + 384, ...), re-reading any word whose tag is
    // not yet current (the count is relaxed), and unpack them into the shared act.  (Starting
    // the reads before the last CTAs count in and re-polling their words cost ~0.9 us.)
    named_sync(kBarConsumers, kConsumerThreads);
    if (tid == 0) {
        red_relaxed_gpu_add(&p.ctl->n_act, 1u);
        if (p.trace) p.trace[cta * kTraceSlots + 11] = globaltimer_ns();
        if (ok1 && !wait_count(&p.ctl->n_act, (uint32_t)G * tag, deadline)) {
            atomicExch(&p.ctl->status, (uint32_t)MMRS_ERR_TIMEOUT);
            s.ctl[kCtlFail] = 1;
        }
    }
    named_sync(kBarConsumers, kConsumerThreads);
    {
        // all of a thread's loads in flight at once (kActWords per pass), then one check of their
        // tags; a word from before this launch (the count is relaxed) sends the thread through
        // the compact path that re-polls each word
        const int nwords = 9 * (nvs * I / 32);
        auto unpack = [&](unsigned long long v, int wi) {
            const int b = wi / 9, j = wi - 9 * b;
            if (j < 8) {
                *reinterpret_cast<uint32_t *>(s.aq_s + act_swz(32 * b + 4 * j)) = (uint32_t)v;
            } else {
                s.ad_s[b] = __half2float(__ushort_as_half((unsigned short)(v & 0xffffu)));
                s.aS_s[b] = (int)(short)((uint32_t)v >> 16);
            }
        };
        for (int w0 = 0; w0 < nwords && ok1 && !s.ctl[kCtlFail]; w0 += kActWords * kConsumerThreads) {
            unsigned long long v[kActWords];
#pragma unroll
            for (int i = 0; i < kActWords; ++i) {
                const int wi = w0 + tid + i * kConsumerThreads;
                v[i] = wi < nwords ? ld_relaxed_gpu_u64(p.arec + wi) : 0ull;
            }
            bool stale = false;
#pragma unroll
            for (int i = 0; i < kActWords; ++i)
                stale |= w0 + tid + i * kConsumerThreads < nwords && (uint32_t)(v[i] >> 32) != tag;
            if (!stale) {
#pragma unroll
                for (int i = 0; i < kActWords; ++i) {
                    const int wi = w0 + tid + i * kConsumerThreads;
                    if (wi < nwords) unpack(v[i], wi);
                }
                continue;
            }
#pragma unroll 1
            for (int i = 0; i < kActWords; ++i) {
                const int wi = w0 + tid + i * kConsumerThreads;
                if (wi >= nwords) break;
                unsigned long long x = ld_relaxed_gpu_u64(p.arec + wi);
                uint32_t spins = 0;
                while ((uint32_t)(x >> 32) != tag) {
                    if ((++spins & 63u) == 0 && globaltimer_ns() > deadline) {
                        atomicExch(&p.ctl->status, (uint32_t)MMRS_ERR_TIMEOUT);
                        s.ctl[kCtlFail] = 1;
                        break;
                    }
                    x = ld_relaxed_gpu_u64(p.arec + wi);
                }
                unpack(x, wi);
            }
        }
    }
    if (!ok1 && tid == 0) s.ctl[kCtlFail] = 1;
    if (tid == 0 && p.trace) p.trace[cta * kTraceSlots + 5] = globaltimer_ns();
    named_sync(kBarConsumers, kConsumerThreads);
    if (s.ctl[kCtlFail]) aborted = true;
    build_task_scales(s.ats, s.ad_s, s.aS_s, nvs * (I / 64), tid, kConsumerThreads);
    named_sync(kBarConsumers, kConsumerThreads);
    if (tid == 0 && p.trace) p.trace[cta * kTraceSlots + 6] = globaltimer_ns();

    // the next kernel in the stream may start its CTAs as this kernel's CTAs retire
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    // ---- P3: down: lane t takes (position, block) pair t % pairs and rows t / pairs, + slots, ...
    {
        constexpr int BB = DN == MMRS_Q5K ? Q5K_BYTES : Q4K_BYTES;
        const int pairs = nvs * NBd;
        const int slots = pairs > 0 ? kConsumerThreads / pairs : 0;
        const bool d_lane = tid < pairs * slots;
        const int P = d_lane ? tid % pairs : 0, first = d_lane ? tid / pairs : 0;
        const int vp = P / NBd, sb = P % NBd;
        if (d_lane) load_block_act(s.aq_s + (size_t)vp * I + QK_K * sb, P, s.ats + vp * (I / 64) + 4 * sb, act);
        const int k = n_gu_units + vp, st = k % p.stages;
        // A warp's lanes may hold positions a ring apart (the pairs wrap within a warp), so the
        // down lanes take no warp-collective step: each lane computes its rows, then adds its
        // count to the unit's stage once; the lane that completes the unit issues unit k + stages.
        int done_rows = 0;
        for (int r = first; d_lane && r < nres; r += slots) {
            if (done_rows == 0) wait_landed(k, st);
            float v = 0.f;
            if (!aborted) v = block_dot<DN>(s.stages + (size_t)st * p.stage_bytes + (size_t)r * dn_row_bytes + BB * sb, act);
            s.bpart[(vp * nres + r) * NBd + sb] = v;
            ++done_rows;
        }
        if (tid == 0 && p.trace) p.trace[cta * kTraceSlots + 17] = globaltimer_ns();
        if (done_rows > 0) {
            const int old = atom_add_acq_rel_cta(&s.done[st], done_rows);
            if (old + done_rows == nres * NBd) {
                s.done[st] = 0;
                if (k + p.stages < n_units && !aborted) issue(k + p.stages);
            }
        }
        __syncwarp();
    }

    // ---- y = fixed 8-way tree over the routed experts (moe_gguf.cu:328-342) + residual ---------
    named_sync(kBarConsumers, kConsumerThreads);
    // expert row of slot j for output row r, weighted by the route weight (0 for a slot not
    // computed here), one (row, slot) per thread; then the 8-way tree per row
    for (int t = tid; t < nres * kTopK; t += kConsumerThreads) {
        const int r = t / kTopK, j = t % kTopK, vp = s.posof[j];
        s.dn_acc[t] = vp >= 0 ? sum_blocks(s.bpart + (vp * nres + r) * NBd, NBd) * s.w[j] : 0.f;
    }
    named_sync(kBarConsumers, kConsumerThreads);
    if (tid == 0 && p.trace) p.trace[cta * kTraceSlots + 16] = globaltimer_ns();
    auto slot_rows = [&](int r, float (&q)[kTopK]) {
#pragma unroll
        for (int j = 0; j < kTopK; ++j) q[j] = s.dn_acc[r * kTopK + j];
    };
    if (p.world <= 1) {
        for (int r = tid; r < nres && !aborted; r += kConsumerThreads) {
            float q[kTopK];
            slot_rows(r, q);
            float y = ((q[0] + q[4]) + (q[2] + q[6])) + ((q[1] + q[5]) + (q[3] + q[7]));
            if (p.residual) y = y + s.res_s[r];
            p.y[dn_r0 + r] = y;
        }
    } else {
        // Fused exchange of the partial rows with the other ranks over NVLink, pushed: this
        // CTA's rows go to every rank's receive buffer (slot [token & 1][this rank]) as 64-bit
        // words {token, f32 bits}; then each thread waits (bounded) until its rows from every
        // rank carry the token in this rank's own memory, sums them in rank order (bit-identical
        // on all ranks) and adds the residual
        // (TensorParallelRankGroup::all_reduce_sum_with_residual, tensor_parallel.rs:786-812).
        // The token is the group's operation counter: every layer sharing the group draws a fresh
        // one, so a word written for another layer's exchange never satisfies this wait.  The
        // rows are pushed even after a failed wait, so that no peer waits for them in vain.
        const uint32_t token = p.token;
        const unsigned long long hi = (unsigned long long)token << 32;
        const size_t slot = (size_t)(token & 1u) * kMaxRanks;
        for (int r = tid; r < nres; r += kConsumerThreads) {
            float q[kTopK];
            slot_rows(r, q);
            const float v = ((q[0] + q[4]) + (q[2] + q[6])) + ((q[1] + q[5]) + (q[3] + q[7]));
            const unsigned long long w = hi | __float_as_uint(v);
            for (int rk = 0; rk < p.world; ++rk) {
                uint8_t *base = rk == p.rank ? p.xch : p.xpeer[rk];
                st_relaxed_sys_u64(reinterpret_cast<unsigned long long *>(base + kXchDRecv) +
                                   (slot + p.rank) * kXchMaxHidden + dn_r0 + r, w);
            }
        }
        if (tid == 0 && p.trace) p.trace[cta * kTraceSlots + 18] = globaltimer_ns();
        const unsigned long long *recv = reinterpret_cast<const unsigned long long *>(p.xch + kXchDRecv) + slot * kXchMaxHidden;
        const uint64_t xdl = globaltimer_ns() + p.timeout_ns;
        for (int r = tid; r < nres; r += kConsumerThreads) {
            const int row = dn_r0 + r;
            unsigned long long w[kMaxRanks];
#pragma unroll
            for (int rk = 0; rk < kMaxRanks; ++rk)  // all loads in flight before the checks
                w[rk] = rk < p.world ? ld_relaxed_sys_u64(recv + (size_t)rk * kXchMaxHidden + row) : hi;
            bool stale = false;
#pragma unroll
            for (int rk = 0; rk < kMaxRanks; ++rk) stale |= (uint32_t)(w[rk] >> 32) != token;
            float y = 0.f;
            if (!stale) {
                y = __uint_as_float((uint32_t)w[0]);
#pragma unroll
                for (int rk = 1; rk < kMaxRanks; ++rk)
                    if (rk < p.world) y = y + __uint_as_float((uint32_t)w[rk]);
            } else {
                // a rank's row has not arrived yet: poll each rank's word in turn (rank order)
                bool xok = true;
#pragma unroll 1
                for (int rk = 0; rk < p.world && xok; ++rk) {
                    unsigned long long x = ld_relaxed_sys_u64(recv + (size_t)rk * kXchMaxHidden + row);
                    uint32_t spins = 0;
                    while ((uint32_t)(x >> 32) != token) {
                        if ((++spins & 63u) == 0 && globaltimer_ns() > xdl) {
                            atomicExch(&p.ctl->status, (uint32_t)MMRS_ERR_TIMEOUT);
                            atomicExch(reinterpret_cast<uint32_t *>(p.xch + kXchStatus), (uint32_t)MMRS_ERR_TIMEOUT);
                            xok = false;
                            break;
                        }
                        x = ld_relaxed_sys_u64(recv + (size_t)rk * kXchMaxHidden + row);
                    }
                    y = rk == 0 ? __uint_as_float((uint32_t)x) : y + __uint_as_float((uint32_t)x);
                }
                if (!xok) continue;
            }
            if (p.residual) y = y + s.res_s[r];
            p.y[row] = y;
        }
    }
    // No copy may still be landing in shared memory when the CTA retires.  Without a failed wait
    // every issued unit has been waited for by the lanes that computed it; after an expired wait
    // a unit may have been issued and never waited for, so the CTA waits for each stage's last.
    if (tid == 0 && ok1 && s.ctl[kCtlFail]) {
        for (int st = 0; st < p.stages; ++st) {
            const int k = *reinterpret_cast<volatile int *>(&s.ticket[st]);
            if (k >= 0) mbar_wait_bounded(&s.full[st], (uint32_t)(k / p.stages) & 1u, deadline + 1000000000ull);
        }
    }
    if (tid == 0) {
        p.ctl->arrive[cta] = tag;  // this CTA's launch count (read only by this CTA's next launch)
        if (p.trace) p.trace[cta * kTraceSlots + 7] = globaltimer_ns();
    }
}

// ------------------------------------------------------------------------------------------
// Host side
// ------------------------------------------------------------------------------------------
size_t decode_smem_bytes(const DecodeParams &p) {
    auto a16 = [](size_t v) { return (v + 15) / 16 * 16; };
    size_t b = a16((size_t)p.stages * p.stage_bytes) + a16(sizeof(uint64_t) * p.stages);
    b += a16(p.H) + 2 * a16(4 * (p.H / 32)) + a16(16 * (p.H / 64));
    b += a16((size_t)kTopK * p.I) + 2 * a16(4 * kTopK * (p.I / 32)) + a16(16 * kTopK * (p.I / 64));
    b += a16(4 * 16) + a16(8 * 64) + a16(4 * 64) + 5 * a16(4 * kTopK);  // part, cand, csig, slotsig, ids, vslot, posof, w
    b += a16(4 * (size_t)kTopK * p.res_slots);                           // dn_acc
    b += a16(4 * decode_part_floats(p)) + a16(4 * (size_t)p.res_slots);
    b += a16(16 * kMaxUnits) + a16(4 * kMaxUnits) + a16(8 * kMaxUnits) + a16(4 * kMaxUnits) + a16(16 * (size_t)p.act_slots);
    b += 2 * a16(4 * (size_t)p.stages) + a16(4 * kCtlWords);
    return b;
}

int decode_configure(DecodeParams &p, int num_sms, int max_smem) {
    if (p.H % QK_K || p.I % QK_K || p.E < kTopK || p.E > 256 || p.E % 4) return MMRS_ERR_UNSUPPORTED;
    if ((p.gu_type != MMRS_Q4K && p.gu_type != MMRS_Q5K) || (p.dn_type != MMRS_Q4K && p.dn_type != MMRS_Q5K))
        return MMRS_ERR_UNSUPPORTED;
    if (p.H / 8 / 4 > 128) return MMRS_ERR_UNSUPPORTED;  // router slice: at most 4 float4 a lane (H <= 4096)
    // one consumer lane per super-block of a gate/up row, and per (position, block) of the down rows
    if (p.H / QK_K > kConsumerThreads || kTopK * (p.I / QK_K) > kConsumerThreads) return MMRS_ERR_UNSUPPORTED;
    p.act_slots = 32 * ((kTopK * p.I / 32 + num_sms - 1) / num_sms) + 1;  // whole Q8_1 blocks a CTA
    p.res_slots = (p.H + num_sms - 1) / num_sms + 1;
    if (p.E > 2 * num_sms || num_sms > kDecodeMaxCtas) return MMRS_ERR_UNSUPPORTED;
    const size_t gu_row = kq_row_bytes(p.gu_type, p.H);
    const size_t dn_stage = kq_row_bytes(p.dn_type, p.I) * (p.res_slots - 1);
    // a gate/up copy unit: as many whole rows as a down unit's stage holds (at least 4)
    p.gu_unit_rows = (int)(dn_stage / gu_row) > 4 ? (int)(dn_stage / gu_row) : 4;
    // table bounds: a CTA's gate/up chunks (one producer lane each; each slot boundary may add one)
    const int max_chunks = (p.act_slots + p.gu_unit_rows - 1) / p.gu_unit_rows + kTopK;
    if (max_chunks > 32 || 2 * max_chunks + kTopK > kMaxUnits || p.gu_unit_rows > 0xffff || p.res_slots > 0xffff)
        return MMRS_ERR_UNSUPPORTED;
    const size_t gu_stage = gu_row * p.gu_unit_rows;
    p.stage_bytes = (int)(((gu_stage > dn_stage ? gu_stage : dn_stage) + 127) / 128 * 128);
    p.stages = 0;
    DecodeParams q = p;
    for (int st = 16; st >= 3; --st) {
        q.stages = st;
        if (decode_smem_bytes(q) <= (size_t)max_smem) {
            p.stages = st;
            break;
        }
    }
    if (p.stages == 0) return MMRS_ERR_UNSUPPORTED;
    p.grid = num_sms;
    return MMRS_OK;
}

template <int GU, int DN>
static int launch_typed(const DecodeParams &p, size_t smem, cudaStream_t stream) {
    // Raise the dynamic shared-memory limit once per device and instantiation (the attribute is
    // per context); call_once keeps concurrent host threads from racing on it.
    static std::once_flag once[64];
    static cudaError_t set_rc[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return MMRS_ERR_LAUNCH;
    std::call_once(once[dev], [dev] {
        int optin = 0;
        cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        set_rc[dev] =
            cudaFuncSetAttribute(moe_decode_fused_kernel<GU, DN>, cudaFuncAttributeMaxDynamicSharedMemorySize, optin);
    });
    if (set_rc[dev] != cudaSuccess) return MMRS_ERR_LAUNCH;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    // Programmatic dependent launch: the CTAs start (router weights in flight) while the previous
    // kernel retires; griddepcontrol.wait in the kernel orders everything that reads its outputs.
    // No cooperative launch: one CTA per SM always fits (grid = SM count, whole-SM shared memory)
    // and every cross-CTA wait is bounded.
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t err = cudaLaunchKernelEx(&cfg, moe_decode_fused_kernel<GU, DN>, p);
    return err == cudaSuccess ? MMRS_OK : MMRS_ERR_LAUNCH;
}

int decode_launch(const DecodeParams &p, cudaStream_t stream) {
    const size_t smem = decode_smem_bytes(p);
    const bool g5 = p.gu_type == MMRS_Q5K, d5 = p.dn_type == MMRS_Q5K;
    if (g5) return d5 ? launch_typed<MMRS_Q5K, MMRS_Q5K>(p, smem, stream) : launch_typed<MMRS_Q5K, MMRS_Q4K>(p, smem, stream);
    return d5 ? launch_typed<MMRS_Q4K, MMRS_Q5K>(p, smem, stream) : launch_typed<MMRS_Q4K, MMRS_Q4K>(p, smem, stream);
}

}  // namespace mmrs
