// Fused single-token MoE block for B200 (sm_100a).
//
// Replaces, in one persistent launch, the reference's decode chain
//   router Linear (fused_moe.rs:267) -> minimax_moe_decode_topk (moe_gguf.cu:34-100)
//   -> quantize_q8_1 -> moe_gate_up_decode_kernel -> quantize_silu_mul_q8_1
//   -> moe_down_decode_kernel (moe_gguf.cu:200-343, 426-567) -> + residual (model.rs:218)
//
// One CTA per SM: 12 consumer warps + 1 producer warp.
//   P0  router GEMV in the canonical order (8 K-slices; the CTA's two experts x 8 slices are 16
//       (expert, slice) pairs over the 13 warps: 32 lane partials, butterfly, fixed slice tree).
//       The router rows are requested before anything else.  Grid barrier #1: one
//       fire-and-forget arrival per CTA.
//   P1  the consumer warps quantise x to Q8_1 while the producer warp waits for barrier #1;
//       eight warps then take 32 experts each (sigmoid, order-preserving selection key, rounds of
//       redux max / min: that warp's top-8) and the producer warp merges the 64 candidates the same
//       way, renormalises the weights and builds the copy table with its 32 lanes.
//   P2  gate/up: the CTA owns a contiguous range of (slot, row) pairs; copy units of up to three
//       warp shares of rows of the gate or the up matrix (one bulk copy each) stream through a
//       ring of shared-memory stages.  Consumer warps claim sub-units (one warp's rows) in unit
//       order from a CTA counter, so a free warp always takes the oldest unclaimed rows; the last
//       finisher of a unit frees its stage.  The producer issues every unit as soon as its stage
//       is free, so the down units (this CTA's output rows of one expert: one contiguous copy
//       each) land in the ring while gate/up is still being computed.
//   P3  the CTA's gate/up range is a whole number of 32-row Q8_1 blocks, so it quantises
//       act = up * silu(gate) of its own blocks (quantize_silu_mul_q8_1 arithmetic) and writes them
//       out; grid barrier #2; one bulk copy brings the whole quantised vector into every CTA; then
//       the down sub-units, weighted by the route weight, the reference's fixed 8-way tree
//       ((v0+v4)+(v2+v6))+((v1+v5)+(v3+v7)) per output row, + residual.
// Lane work unit ("task"): one 64-weight sub-block pair (super-block sb, pair j) of a row: 32 B of
// quants, dp4a against the Q8_1 activation, MMVQ combine of vec_dot_q4_K_q8_1 / _q5_K_
// (gguf.cuh:727-750, 783-813): dall * sum d8*(dot*sc) - dmin * sum d8*sum(q8)*m.
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
constexpr int kRowsPerLane = 2;  // rows a lane group computes per sub-unit (same activation registers)
constexpr int kSubsPerGuUnit = 3;  // gate/up copy unit = 3 warp shares: stages sized by the down units
constexpr int kMaxUnits = 80;
constexpr int kMaxSubs = 256;
constexpr int kTopK = 8;
constexpr int kTPL = 3;  // tasks (64-weight sub-block pairs) per lane
constexpr int kRouterRounds = (16 + kWarps - 1) / kWarps;
// named barriers: consumers; table ready, router partials, barrier #1 passed (all threads);
// routing candidates ready (the eight routing warps + the producer)
constexpr int kBarConsumers = 1, kBarTable = 3, kBarRouter = 4, kBarRoute = 5, kBarCand = 6;
constexpr int kRouteWarps = 8;  // one expert a lane: E <= 256
// control words in shared memory
enum { kCtlUnits, kCtlGuUnits, kCtlSubGu, kCtlSubs, kCtlNext, kCtlPositions, kCtlOk, kCtlFail, kCtlWords };

// Q8_1 activation in shared memory: q int8 [K] and, per 64-element pair (task), the float4
// {d8 lo block, d8 hi block, d8*sum(q) lo, d8*sum(q) hi}.
struct ActView {
    const int8_t *q;
    const float4 *ts;
};

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

// Per-lane register copy of one task's activation: 64 int8 (lo block, hi block) and the scale
// record {d8 lo, d8 hi, d8*sum(q) lo, d8*sum(q) hi}.
struct TaskAct {
    int lo[8], hi[8];
    float4 ts;
};

__device__ __forceinline__ void load_task_acts(const ActView &a, int lig, int L, int ntasks, TaskAct (&ta)[kTPL]) {
#pragma unroll
    for (int i = 0; i < kTPL; ++i) {
        const int tau = lig + L * i;
        if (tau < ntasks) {
            const int4 *q = reinterpret_cast<const int4 *>(a.q + 64 * tau);
            const int4 a0 = q[0], a1 = q[1], a2 = q[2], a3 = q[3];
            ta[i].lo[0] = a0.x; ta[i].lo[1] = a0.y; ta[i].lo[2] = a0.z; ta[i].lo[3] = a0.w;
            ta[i].lo[4] = a1.x; ta[i].lo[5] = a1.y; ta[i].lo[6] = a1.z; ta[i].lo[7] = a1.w;
            ta[i].hi[0] = a2.x; ta[i].hi[1] = a2.y; ta[i].hi[2] = a2.z; ta[i].hi[3] = a2.w;
            ta[i].hi[4] = a3.x; ta[i].hi[5] = a3.y; ta[i].hi[6] = a3.z; ta[i].hi[7] = a3.w;
            ta[i].ts = a.ts[tau];
        } else {
#pragma unroll
            for (int c = 0; c < 8; ++c) ta[i].lo[c] = ta[i].hi[c] = 0;
            ta[i].ts = make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
}

template <int TYPE>
__device__ __forceinline__ float task_dot(const uint8_t *row, int tau, const TaskAct &a) {
    constexpr int BB = TYPE == MMRS_Q5K ? Q5K_BYTES : Q4K_BYTES;
    const int sb = tau >> 2, j = tau & 3;
    const uint8_t *blk = row + sb * BB;
    const uint4 hdr = *reinterpret_cast<const uint4 *>(blk);
    int d[4] = {0, 0, 0, 0};
    if (TYPE == MMRS_Q5K) {
        const uint4 q0 = *reinterpret_cast<const uint4 *>(blk + 48 + 32 * j);
        const uint4 q1 = *reinterpret_cast<const uint4 *>(blk + 64 + 32 * j);
        const uint4 h0 = *reinterpret_cast<const uint4 *>(blk + 16);
        const uint4 h1 = *reinterpret_cast<const uint4 *>(blk + 32);
        const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
        const uint32_t h[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
        const int rl = (4 - 2 * j) & 31, rh = (3 - 2 * j) & 31;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            const uint32_t lo = (w[c] & 0x0F0F0F0Fu) | (__funnelshift_l(h[c], h[c], rl) & 0x10101010u);
            const uint32_t hi = ((w[c] >> 4) & 0x0F0F0F0Fu) | (__funnelshift_l(h[c], h[c], rh) & 0x10101010u);
            d[c & 1] = __dp4a((int)lo, a.lo[c], d[c & 1]);
            d[2 + (c & 1)] = __dp4a((int)hi, a.hi[c], d[2 + (c & 1)]);
        }
        d[2] += d[3];
    } else {
        const uint4 q0 = *reinterpret_cast<const uint4 *>(blk + 16 + 32 * j);
        const uint4 q1 = *reinterpret_cast<const uint4 *>(blk + 32 + 32 * j);
        const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            d[c & 1] = dp4a_us(w[c] & 0x0F0F0F0Fu, a.lo[c], d[c & 1]);
            d[2 + (c & 1)] = dp4a_us(w[c] & 0xF0F0F0F0u, a.hi[c], d[2 + (c & 1)]);
        }
        d[2] = (d[2] + d[3]) >> 4;  // every high-nibble term carries a factor 16: exact
    }
    const int dlo = d[0] + d[1], dhi = d[2];
    uint32_t scp, mp;
    scale_pair(hdr, j, scp, mp);
    // |d * sc| < 2^22 for Q4_K (32 * 15 * 127 * 63); Q5_K products reach 2^23 and use the plain conversion
    const int plo = dlo * (int)(scp & 0xffu), phi = dhi * (int)(scp >> 8);
    const float flo = TYPE == MMRS_Q5K ? (float)plo : int22_to_float(plo);
    const float fhi = TYPE == MMRS_Q5K ? (float)phi : int22_to_float(phi);
    const float sd = a.ts.x * flo + a.ts.y * fhi;
    const float sm = a.ts.z * small_uint_to_float(mp & 0xffu) + a.ts.w * small_uint_to_float(mp >> 8);
    const float2 dm = __half22float2(*reinterpret_cast<const __half2 *>(&hdr.x));
    return dm.x * sd - dm.y * sm;
}

// Dot of one row (in shared memory) over the lane's tasks tau = lig + L*i.
template <int TYPE>
__device__ __forceinline__ float row_dot(const uint8_t *row, int lig, int L, int ntasks, const TaskAct (&ta)[kTPL]) {
    float v = 0.f;
#pragma unroll
    for (int i = 0; i < kTPL; ++i) {
        const int tau = lig + L * i;
        if (tau < ntasks) v += task_dot<TYPE>(row, tau, ta[i]);
    }
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
// moe_gguf.cu:255-284).  Writes q, and per block the fp16-rounded scale d and the sum of quants S.
__device__ __forceinline__ void quant128(float4 v, int8_t *q, float *d, int *S, int lane) {
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
    reinterpret_cast<int *>(q)[lane] = (q0 & 0xff) | ((q1 & 0xff) << 8) | ((q2 & 0xff) << 16) | ((q3 & 0xff) << 24);
    int s = q0 + q1 + q2 + q3;
#pragma unroll
    for (int m = 4; m > 0; m >>= 1) s += __shfl_xor_sync(0xffffffffu, s, m);
    if ((lane & 7) == 0) {
        d[lane >> 3] = __half2float(__float2half_rn(dd));
        S[lane >> 3] = s;
    }
}

// One Q8_1 block of 32 values, lane l holding value l: the quant128 arithmetic (d = amax/127,
// q = roundf(v/d), fp16-rounded d, sum of quants).
__device__ __forceinline__ void quant32(float v, int8_t *q, float *d, int *S, int lane) {
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
    q[lane] = (int8_t)qi;
    int sq = qi;
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, m);
    if (lane == 0) {
        *d = __half2float(__float2half_rn(dd));
        *S = sq;
    }
}

// The CTA's gate/up range of (position, row) pairs: whole Q8_1 blocks of 32 rows, so that every
// block of act is quantised by the one CTA that computed it.
__device__ __forceinline__ void gu_range(int cta, int G, int nvs, int I, int &p0, int &p1) {
    const int nblk = nvs * I / 32;
    p0 = 32 * (int)((int64_t)cta * nblk / G);
    p1 = 32 * (int)((int64_t)(cta + 1) * nblk / G);
}

// Per-task scale records from per-block (d, S) arrays: nt tasks, 2 blocks each.
__device__ __forceinline__ void build_task_scales(float4 *ts, const float *d, const int *S, int nt, int tid, int nthr) {
    for (int t = tid; t < nt; t += nthr) {
        const float dl = d[2 * t], dh = d[2 * t + 1];
        ts[t] = make_float4(dl, dh, dl * (float)S[2 * t], dh * (float)S[2 * t + 1]);
    }
}

// Bounded wait until unit k has landed in stage st: first the stage's ticket (the producer has
// issued unit k there; a warp may claim unit k before unit k - stages has been issued), then the
// phase of the stage's full barrier.
__device__ __forceinline__ bool wait_unit(uint64_t *full, const int *ticket, int k, int st, int stages,
                                          uint64_t deadline) {
    uint32_t spins = 0;
    while (*reinterpret_cast<const volatile int *>(&ticket[st]) != k) {
        __nanosleep(32);
        if ((++spins & 255u) == 0 && globaltimer_ns() > deadline) return false;
    }
    return mbar_wait_sleep(&full[st], (uint32_t)(k / stages) & 1u, deadline);
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
struct DecodeSmem {
    uint8_t *stages;
    uint64_t *full;
    uint64_t *abar;            // the quantised act copy after barrier #2
    int8_t *xq;                // [H]
    float *xd;                 // [H/32]
    int *xS;                   // [H/32]
    float4 *xts;               // [H/64]
    int8_t *aq_s;              // [8][I] (positions)
    float *ad_s;               // [8][I/32]
    int *aS_s;                 // [8][I/32]
    float4 *ats;               // [8][I/64]
    float *part;               // router slice sums [2][8]
    float *sig;                // [E] sigmoid of the router logits
    uint32_t *cand;            // [2][64] routing candidates: keys, then expert ids
    int *ids;                  // [8] expert of each slot (-1: none, or another rank's)
    int *vslot;                // [8] slot of each position (the computed slots in order)
    float *w;                  // [8]
    float *dn_acc;             // [res_slots][8] weighted expert rows of this CTA's output range
    float *gval, *uval;        // [act_slots] gate / up row values of this CTA's (position, row) range
    float *res_s;              // [res_slots]
    int4 *units;               // [kMaxUnits]
    int *unit_off;             // [kMaxUnits] first row of a gate/up unit in the CTA's range
    int *unit_nsub;            // [kMaxUnits] sub-units of the unit
    const uint8_t **usrc;      // [kMaxUnits] global source of the unit's copy
    uint32_t *ubytes;          // [kMaxUnits] its size
    int2 *subs;                // [kMaxSubs]
    int *ticket;               // [stages] unit last issued into each stage
    int *done;                 // [stages] sub-units of the stage's unit finished
    int *ctl;                  // [kCtlWords]
};

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
    const int dn_r0 = (int)((int64_t)cta * H / G), dn_r1 = (int)((int64_t)(cta + 1) * H / G);
    const int nres = dn_r1 - dn_r0;

    // ---- P0 loads first: the CTA's router rows and the matching x slices ---------------------
    const int slice = H / 8, groups = slice / 4;
    float4 xx[kRouterRounds][4], wv[kRouterRounds][4];
#pragma unroll
    for (int r = 0; r < kRouterRounds; ++r) {
        const int pi = warp + kWarps * r, sl = pi & 7, le = pi >> 3;
        const int e = cta + G * le;
        if (pi < 16 && p.internal_routing && e < E) {
            const float4 *xs = reinterpret_cast<const float4 *>(p.x + sl * slice);
            const float4 *wr = reinterpret_cast<const float4 *>(p.router + (size_t)e * H + sl * slice);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int g = lane + 32 * i;
                if (g < groups) {
                    wv[r][i] = __ldg(wr + g);
                    xx[r][i] = __ldg(xs + g);
                }
            }
        }
    }
    // this CTA's launch count (2 per completed launch: the grid barriers' targets)
    uint32_t epoch = 0;
    if (lane == 0 && (warp == 0 || warp == kProducerWarp)) epoch = __ldcg(&p.ctl->epoch[cta]);
    if (tid == 0 && p.trace) p.trace[cta * 16 + 0] = t_start;

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
        s.abar = reinterpret_cast<uint64_t *>(take(sizeof(uint64_t)));
        s.xq = reinterpret_cast<int8_t *>(take(H));
        s.xd = reinterpret_cast<float *>(take(sizeof(float) * (H / 32)));
        s.xS = reinterpret_cast<int *>(take(sizeof(int) * (H / 32)));
        s.xts = reinterpret_cast<float4 *>(take(sizeof(float4) * (H / 64)));
        s.aq_s = reinterpret_cast<int8_t *>(take((size_t)kTopK * I));
        s.ad_s = reinterpret_cast<float *>(take(sizeof(float) * kTopK * (I / 32)));
        s.aS_s = reinterpret_cast<int *>(take(sizeof(int) * kTopK * (I / 32)));
        s.ats = reinterpret_cast<float4 *>(take(sizeof(float4) * kTopK * (I / 64)));
        s.part = reinterpret_cast<float *>(take(sizeof(float) * 16));
        s.sig = reinterpret_cast<float *>(take(sizeof(float) * 256));
        s.cand = reinterpret_cast<uint32_t *>(take(sizeof(uint32_t) * 128));
        s.ids = reinterpret_cast<int *>(take(sizeof(int) * kTopK));
        s.vslot = reinterpret_cast<int *>(take(sizeof(int) * kTopK));
        s.w = reinterpret_cast<float *>(take(sizeof(float) * kTopK));
        s.dn_acc = reinterpret_cast<float *>(take(sizeof(float) * p.res_slots * kTopK));
        s.gval = reinterpret_cast<float *>(take(sizeof(float) * p.act_slots));
        s.uval = reinterpret_cast<float *>(take(sizeof(float) * p.act_slots));
        s.res_s = reinterpret_cast<float *>(take(sizeof(float) * p.res_slots));
        s.units = reinterpret_cast<int4 *>(take(sizeof(int4) * kMaxUnits));
        s.unit_off = reinterpret_cast<int *>(take(sizeof(int) * kMaxUnits));
        s.unit_nsub = reinterpret_cast<int *>(take(sizeof(int) * kMaxUnits));
        s.usrc = reinterpret_cast<const uint8_t **>(take(sizeof(void *) * kMaxUnits));
        s.ubytes = reinterpret_cast<uint32_t *>(take(sizeof(uint32_t) * kMaxUnits));
        s.subs = reinterpret_cast<int2 *>(take(sizeof(int2) * kMaxSubs));
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
        mbar_init(s.abar, 1);
        fence_mbar_init();
        for (int i = 0; i < kCtlWords; ++i) s.ctl[i] = 0;
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
    if (p.internal_routing && tid < 2) {
        const int ee = cta + G * tid;
        if (ee < E) {
            const float *q = s.part + tid * 8;
            p.logits[ee] = ((q[0] + q[1]) + (q[2] + q[3])) + ((q[4] + q[5]) + (q[6] + q[7]));
        }
    }
    named_sync(kBarRouter, kThreads);  // both logits written before the release below
    if (tid == 0) {
        if (p.trace) p.trace[cta * 16 + 1] = globaltimer_ns();
        // grid barrier #1 arrival (fire and forget); the producer warp waits for the count
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(&p.ctl->count) : "memory");
    }

    const size_t gu_row_bytes = kq_row_bytes(p.gu_type, H);
    const size_t dn_row_bytes = kq_row_bytes(p.dn_type, I);
    const size_t gu_expert_bytes = gu_row_bytes * I;
    const size_t dn_expert_bytes = dn_row_bytes * H;
    const int Lg = p.gu_lanes, Ld = p.dn_lanes;
    const int gu_sub = p.gu_sub_rows, dn_sub = p.dn_sub_rows, U_gu = p.gu_unit_rows;

    // Issue copy unit k into ring stage k % stages (one thread).  The first `stages` units are
    // issued by the producer warp once the table is built; every later unit by the warp that
    // finishes the last sub-unit of unit k - stages, which frees that stage.
    auto issue = [&](int k) {
        const int st = k % p.stages;
        *reinterpret_cast<volatile int *>(&s.ticket[st]) = k;
        const uint32_t bytes = s.ubytes[k];
        if (p.trace) {
            if (k == 0) p.trace[cta * 16 + 8] = globaltimer_ns();
            if (k == s.ctl[kCtlGuUnits]) p.trace[cta * 16 + 10] = globaltimer_ns();
            if (k == s.ctl[kCtlUnits] - 1) p.trace[cta * 16 + 9] = globaltimer_ns();
        }
        mbar_arrive_expect_tx_sink(&s.full[st], bytes);
        bulk_g2s(s.stages + (size_t)st * p.stage_bytes, s.usrc[k], bytes, &s.full[st]);
    };

    if (warp == kProducerWarp) {
        // ================================ producer warp ===================================
        bool ok = true;
        if (lane == 0) {
            const uint32_t target = (uint32_t)G * (epoch + 1u);
            uint32_t spins = 0;
            while ((int)(ld_acquire_gpu(&p.ctl->count) - target) < 0) {
                __nanosleep(16);
                if ((++spins & 255u) == 0 && globaltimer_ns() > deadline) {
                    atomicExch(&p.ctl->status, (uint32_t)MMRS_ERR_TIMEOUT);
                    ok = false;
                    break;
                }
            }
            if (p.trace) p.trace[cta * 16 + 2] = globaltimer_ns();
        }
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (lane == 0) s.ctl[kCtlOk] = ok ? 1 : 0;
        __syncwarp();
        named_arrive(kBarRoute, kThreads);  // barrier #1 passed: the routing warps may read the logits
        named_sync(kBarCand, 32 * (kRouteWarps + 1));
        // ---- merge of the routing warps' candidates (8 per warp, each warp's in rank order) --------
        int slot_id = -1;  // lane k < 8: expert of slot k
        float slot_w = 0.f;
        if (p.internal_routing) {
            if (ok) {
                const int nc = 8 * ((E + 31) / 32);
                const uint32_t ka = lane < nc ? s.cand[lane] : 0u, ia = lane < nc ? s.cand[64 + lane] : 0xffffffffu;
                const uint32_t kb = lane + 32 < nc ? s.cand[lane + 32] : 0u;
                const uint32_t ib = lane + 32 < nc ? s.cand[64 + lane + 32] : 0xffffffffu;
                bool ta = false, tb = false;
#pragma unroll
                for (int k = 0; k < kTopK; ++k) {
                    // larger key first, lower expert id among equal keys (the stable descending order)
                    const uint32_t mk = __reduce_max_sync(0xffffffffu, max(ta ? 0u : ka, tb ? 0u : kb));
                    const uint32_t ca = (!ta && ka == mk) ? ia : 0xffffffffu;
                    const uint32_t cb = (!tb && kb == mk) ? ib : 0xffffffffu;
                    const uint32_t me = __reduce_min_sync(0xffffffffu, min(ca, cb));
                    if (ca == me) ta = true;
                    else if (cb == me) tb = true;
                    if (lane == k) slot_id = (int)me;
                }
                // weights: sig / ((v0+v4)+(v2+v6))+((v1+v5)+(v3+v7)), lane k keeps w_k
                const float my_sig = lane < kTopK ? s.sig[slot_id] : 0.f;
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
        // ---- positions: the computed slots in order (expert parallel: this rank's only) ------
        const bool compact = p.world > 1 && p.ep;
        int id = (ok && lane < kTopK) ? slot_id : -1;
        if (compact && id >= 0 && id % p.world != p.rank) id = -1;
        const bool keep = lane < kTopK && id >= 0;
        const uint32_t kept = __ballot_sync(0xffffffffu, keep);
        const int nvs = __popc(kept);
        if (lane < kTopK) {
            s.ids[lane] = id;
            s.w[lane] = slot_w;
            if (keep) s.vslot[__popc(kept & ((1u << lane) - 1u))] = lane;
        }
        __syncwarp();
        // ---- copy table: lane c computes gate/up chunk c of the CTA's (position, row) range --
        int gu_p0, gu_p1;
        gu_range(cta, G, nvs, I, gu_p0, gu_p1);
        int n_chunks = 0, c_left = lane, my_pos = -1, my_row0 = 0, my_n = 0, my_off = 0;
        for (int pos = gu_p0 / I, q = gu_p0; q < gu_p1; ++pos) {
            const int seg_end = min(gu_p1, (pos + 1) * I);
            const int nc = (seg_end - q + U_gu - 1) / U_gu;
            if (c_left >= 0 && c_left < nc) {
                const int r = q + c_left * U_gu;
                my_pos = pos;
                my_row0 = r - pos * I;
                my_n = min(U_gu, seg_end - r);
                my_off = r - gu_p0;
            }
            c_left -= nc;
            n_chunks += nc;
            q = seg_end;
        }
        const int n_gu_units = 2 * n_chunks;
        const int ns = my_pos >= 0 ? (my_n + gu_sub - 1) / gu_sub : 0;
        int incl = ns;  // inclusive prefix of sub-units over chunks
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += t;
        }
        const int base = 2 * (incl - ns);  // gate and up sub-units of the earlier chunks
        const int n_sub_gu = 2 * __shfl_sync(0xffffffffu, incl, 31);
        if (my_pos >= 0) {
            for (int h = 0; h < 2; ++h) {
                const int k = 2 * lane + h;
                s.units[k] = make_int4(h, my_pos, my_row0, my_n);
                s.unit_off[k] = my_off;
                s.unit_nsub[k] = ns;
                const int e = s.ids[s.vslot[my_pos]];
                s.usrc[k] = (h == 0 ? p.gate : p.up) + (size_t)e * gu_expert_bytes + (size_t)my_row0 * gu_row_bytes;
                s.ubytes[k] = (uint32_t)(gu_row_bytes * my_n);
                for (int j = 0; j < ns; ++j) {
                    const int r0 = j * gu_sub;
                    s.subs[base + h * ns + j] = make_int2(k, r0 | (min(gu_sub, my_n - r0) << 16));
                }
            }
        }
        // down units: one per position, all of this CTA's output rows
        const int nsd = nres > 0 ? (nres + dn_sub - 1) / dn_sub : 0;
        const int n_dn_units = nsd > 0 ? nvs : 0;
        if (lane < n_dn_units) {
            const int k = n_gu_units + lane;
            s.units[k] = make_int4(2, lane, dn_r0, nres);
            s.unit_off[k] = 0;
            s.unit_nsub[k] = nsd;
            const int e = s.ids[s.vslot[lane]];
            s.usrc[k] = p.down + (size_t)e * dn_expert_bytes + (size_t)dn_r0 * dn_row_bytes;
            s.ubytes[k] = (uint32_t)(dn_row_bytes * nres);
            for (int j = 0; j < nsd; ++j) {
                const int r0 = j * dn_sub;
                s.subs[n_sub_gu + lane * nsd + j] = make_int2(k, r0 | (min(dn_sub, nres - r0) << 16));
            }
        }
        if (lane == 0) {
            s.ctl[kCtlUnits] = n_gu_units + n_dn_units;
            s.ctl[kCtlGuUnits] = n_gu_units;
            s.ctl[kCtlSubGu] = n_sub_gu;
            s.ctl[kCtlSubs] = n_sub_gu + n_dn_units * nsd;
            s.ctl[kCtlPositions] = nvs;
            s.ctl[kCtlOk] = ok ? 1 : 0;
            if (p.trace) p.trace[cta * 16 + 3] = globaltimer_ns();
        }
        __syncwarp();
        named_arrive(kBarTable, kThreads);  // table complete: the consumers may claim
        __syncwarp();
        // ---- first ring fill (lane 0); later units are issued by the consumer warps -------------
        if (lane == 0 && ok) {
            const int n = min(n_gu_units + n_dn_units, p.stages);
            for (int k = 0; k < n; ++k) issue(k);
        }
        return;
    }

    // ================================ consumer warps ======================================
    // While the producer waits for barrier #1 and routes: Q8_1 of x, residual, zeroed sums.
    {
        const int nxc = H / 128;
        for (int c = warp; c < nxc; c += kConsumerWarps) {
            const float4 xv = __ldg(reinterpret_cast<const float4 *>(p.x) + c * 32 + lane);
            quant128(xv, s.xq + c * 128, s.xd + c * 4, s.xS + c * 4, lane);
        }
        for (int r = tid; r < nres; r += kConsumerThreads) s.res_s[r] = p.residual ? __ldg(p.residual + dn_r0 + r) : 0.f;
        for (int i = tid; i < nres * kTopK; i += kConsumerThreads) s.dn_acc[i] = 0.f;
        named_sync(kBarConsumers, kConsumerThreads);
        build_task_scales(s.xts, s.xd, s.xS, H / 64, tid, kConsumerThreads);
    }
    named_sync(kBarRoute, kThreads);  // grid barrier #1 passed (the producer polled it)
    if (warp < kRouteWarps) {
        // sigmoid, selection score as an order-preserving key, and this warp's top-8 of its 32
        // experts by rounds of redux max (key) and redux min (id among the lanes holding it)
        const int e = 32 * warp + lane;
        if (p.internal_routing && s.ctl[kCtlOk] && 32 * warp < E) {
            uint32_t key = 0u;  // experts >= E are never selected (E >= 8 real keys are > 0)
            if (e < E) {
                const float sg = __fdiv_rn(1.0f, 1.0f + expf(-__ldcg(p.logits + e)));
                s.sig[e] = sg;
                key = sel_key(sg, __ldg(p.bias + e));
            }
            bool taken = false;
#pragma unroll
            for (int k = 0; k < kTopK; ++k) {
                const uint32_t mk = __reduce_max_sync(0xffffffffu, taken ? 0u : key);
                const uint32_t me = __reduce_min_sync(0xffffffffu, (!taken && key == mk) ? (uint32_t)e : 0xffffffffu);
                taken |= (uint32_t)e == me;
                if (lane == 0) {
                    s.cand[8 * warp + k] = mk;
                    s.cand[64 + 8 * warp + k] = me;
                }
            }
        }
        named_arrive(kBarCand, 32 * (kRouteWarps + 1));
    }
    named_sync(kBarTable, kThreads);
    const bool ok1 = s.ctl[kCtlOk] != 0;
    const int n_sub_gu = s.ctl[kCtlSubGu], n_sub = s.ctl[kCtlSubs], nvs = s.ctl[kCtlPositions];
    const int n_units = s.ctl[kCtlUnits];
    bool aborted = !ok1;
    auto claim = [&]() -> int {
        int v = 0;
        if (lane == 0) v = atomicAdd(&s.ctl[kCtlNext], 1);
        return __shfl_sync(0xffffffffu, v, 0);
    };
    // A warp that finished a sub-unit of unit k: the last finisher (its acquire covers the other
    // warps' reads of the stage) issues unit k + stages into the freed stage.
    auto finish = [&](int k, int st) {
        __syncwarp();
        if (lane == 0) {
            const int old = atom_add_acq_rel_cta(&s.done[st], 1);
            if (old + 1 == s.unit_nsub[k]) {
                s.done[st] = 0;
                if (k + p.stages < n_units && !aborted) issue(k + p.stages);
            }
        }
    };

    // ---- P2: gate / up sub-units ----------------------------------------------------------------
    int g = claim();
    {
        const int ntasks = (H / QK_K) * 4;
        const int lgi = lane / Lg, lig = lane % Lg;
        TaskAct ta[kTPL];
        load_task_acts(ActView{s.xq, s.xts}, lig, Lg, ntasks, ta);
        while (g < n_sub_gu) {
            const int2 su = s.subs[g];
            const int k = su.x, ro = su.y & 0xffff, nr = su.y >> 16;
            const int4 u = s.units[k];
            const int st = k % p.stages;
            if (!aborted && !wait_unit(s.full, s.ticket, k, st, p.stages, deadline)) {
                atomicExch(&p.ctl->status, (uint32_t)MMRS_ERR_TIMEOUT);
                aborted = true;
            }
            const int rA = ro + lgi * kRowsPerLane, rB = rA + 1, rend = ro + nr;
            float vA = 0.f, vB = 0.f;
            if (!aborted && rA < rend) {
                const uint8_t *base = s.stages + (size_t)st * p.stage_bytes;
                const uint8_t *rowA = base + (size_t)rA * gu_row_bytes;
                const uint8_t *rowB = base + (size_t)min(rB, rend - 1) * gu_row_bytes;
                vA = row_dot<GU>(rowA, lig, Lg, ntasks, ta);
                vB = row_dot<GU>(rowB, lig, Lg, ntasks, ta);
            }
#pragma unroll
            for (int m = 16; m > 0; m >>= 1)
                if (m < Lg) {
                    vA += __shfl_xor_sync(0xffffffffu, vA, m);
                    vB += __shfl_xor_sync(0xffffffffu, vB, m);
                }
            if (lig == 0) {
                float *gv = (u.x == 0 ? s.gval : s.uval) + s.unit_off[k];
                if (rA < rend) gv[rA] = vA;
                if (rB < rend) gv[rB] = vB;
            }
            finish(k, st);
            g = claim();
        }
    }

    // ---- P3: Q8_1 of act for the CTA's blocks, grid barrier #2, copy of the whole vector ---------
    named_sync(kBarConsumers, kConsumerThreads);  // every gate/up sub-unit of this CTA is done
    if (tid == 0 && p.trace) p.trace[cta * 16 + 4] = globaltimer_ns();
    {
        int gu_p0, gu_p1;
        gu_range(cta, G, nvs, I, gu_p0, gu_p1);
        for (int i = tid; i < gu_p1 - gu_p0; i += kConsumerThreads) {
            const float gv = s.gval[i];
            // act = up * silu(gate) (moe_gguf.cu:272-273), in place of the gate values
            s.gval[i] = s.uval[i] * __fdiv_rn(gv, 1.0f + expf(-gv));
        }
        named_sync(kBarConsumers, kConsumerThreads);
        // quantize_silu_mul_q8_1 (moe_gguf.cu:255-284): one warp per block of 32 rows
        for (int b = gu_p0 / 32 + warp; b < gu_p1 / 32 && !aborted; b += kConsumerWarps)
            quant32(s.gval[32 * b - gu_p0 + lane], p.aq + 32 * b, p.ad + b, p.aS + b, lane);
    }
    named_sync(kBarConsumers, kConsumerThreads);
    if (tid == 0) {
        bool ok2 = ok1;
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(&p.ctl->count) : "memory");
        const uint32_t target = (uint32_t)G * (epoch + 2u);
        uint32_t spins = 0;
        while (ok2 && (int)(ld_acquire_gpu(&p.ctl->count) - target) < 0) {
            __nanosleep(16);
            if ((++spins & 255u) == 0 && globaltimer_ns() > deadline) {
                atomicExch(&p.ctl->status, (uint32_t)MMRS_ERR_TIMEOUT);
                ok2 = false;
            }
        }
        if (ok2) p.ctl->epoch[cta] = epoch + 2u;  // read again only by this CTA's next launch
        if (p.trace) p.trace[cta * 16 + 5] = globaltimer_ns();
        // the whole quantised act [positions][I] (+ scales, sums) in one bulk copy per array; the
        // other CTAs' generic writes are ordered before these async-proxy reads
        bool copied = false;
        if (ok2 && nvs > 0) {
            const uint32_t qb = (uint32_t)(nvs * I), sb = (uint32_t)(sizeof(float) * nvs * (I / 32));
            asm volatile("fence.proxy.async;" ::: "memory");
            mbar_arrive_expect_tx(s.abar, qb + 2 * sb);
            bulk_g2s(s.aq_s, p.aq, qb, s.abar);
            bulk_g2s(s.ad_s, p.ad, sb, s.abar);
            bulk_g2s(s.aS_s, p.aS, sb, s.abar);
            copied = true;
        }
        if (copied && !mbar_wait_bounded(s.abar, 0u, deadline + 1000000000ull)) {
            atomicExch(&p.ctl->status, (uint32_t)MMRS_ERR_TIMEOUT);
            ok2 = false;
        }
        s.ctl[kCtlFail] = ok2 ? 0 : 1;
    }
    named_sync(kBarConsumers, kConsumerThreads);
    if (s.ctl[kCtlFail]) aborted = true;
    build_task_scales(s.ats, s.ad_s, s.aS_s, nvs * (I / 64), tid, kConsumerThreads);
    named_sync(kBarConsumers, kConsumerThreads);
    if (tid == 0 && p.trace) p.trace[cta * 16 + 6] = globaltimer_ns();

    // ---- P3: down sub-units -------------------------------------------------------------------
    {
        const int ntasks = (I / QK_K) * 4;
        const int lgi = lane / Ld, lig = lane % Ld;
        TaskAct ta[kTPL];
        int cur_vp = -1;
        while (g < n_sub) {
            const int2 su = s.subs[g];
            const int k = su.x, ro = su.y & 0xffff, nr = su.y >> 16;
            const int4 u = s.units[k];
            const int st = k % p.stages;
            const int vp = u.y, slot = s.vslot[vp];
            if (vp != cur_vp) {
                load_task_acts(ActView{s.aq_s + (size_t)vp * I, s.ats + vp * (I / 64)}, lig, Ld, ntasks, ta);
                cur_vp = vp;
            }
            if (!aborted && !wait_unit(s.full, s.ticket, k, st, p.stages, deadline)) {
                atomicExch(&p.ctl->status, (uint32_t)MMRS_ERR_TIMEOUT);
                aborted = true;
            }
            const int rA = ro + lgi * kRowsPerLane, rB = rA + 1, rend = ro + nr;
            float vA = 0.f, vB = 0.f;
            if (!aborted && rA < rend) {
                const uint8_t *base = s.stages + (size_t)st * p.stage_bytes;
                const uint8_t *rowA = base + (size_t)rA * dn_row_bytes;
                const uint8_t *rowB = base + (size_t)min(rB, rend - 1) * dn_row_bytes;
                vA = row_dot<DN>(rowA, lig, Ld, ntasks, ta);
                vB = row_dot<DN>(rowB, lig, Ld, ntasks, ta);
            }
#pragma unroll
            for (int m = 16; m > 0; m >>= 1)
                if (m < Ld) {
                    vA += __shfl_xor_sync(0xffffffffu, vA, m);
                    vB += __shfl_xor_sync(0xffffffffu, vB, m);
                }
            if (lig == 0) {
                const float wslot = s.w[slot];
                if (rA < rend) s.dn_acc[rA * kTopK + slot] = vA * wslot;
                if (rB < rend) s.dn_acc[rB * kTopK + slot] = vB * wslot;
            }
            finish(k, st);
            g = claim();
        }
    }

    // ---- y = fixed 8-way tree over the routed experts (moe_gguf.cu:328-342) + residual ---------
    named_sync(kBarConsumers, kConsumerThreads);
    if (p.world <= 1) {
        for (int r = tid; r < nres && !aborted; r += kConsumerThreads) {
            const float *q = s.dn_acc + r * kTopK;
            float y = ((q[0] + q[4]) + (q[2] + q[6])) + ((q[1] + q[5]) + (q[3] + q[7]));
            if (p.residual) y = y + s.res_s[r];
            p.y[dn_r0 + r] = y;
        }
    } else {
        // Fused exchange of the partial rows with the other ranks over NVLink: publish this
        // CTA's rows in the exchange region (buffer token & 1), release a per-CTA flag, wait
        // (bounded) for the same CTA's flag on every peer, then sum the ranks' rows in rank
        // order (bit-identical on all ranks) and add the residual
        // (TensorParallelRankGroup::all_reduce_sum_with_residual, tensor_parallel.rs:786-812).
        // The token is the group's operation counter: every layer sharing the group draws a
        // fresh one, so a flag raised for another layer's exchange never satisfies this wait.
        const uint32_t token = p.token;
        const size_t part_off = kXchDPart + sizeof(float) * (size_t)(token & 1u) * kXchMaxHidden;
        float *mine = reinterpret_cast<float *>(p.xch + part_off);
        for (int r = tid; r < nres; r += kConsumerThreads) {
            const float *q = s.dn_acc + r * kTopK;
            mine[dn_r0 + r] = ((q[0] + q[4]) + (q[2] + q[6])) + ((q[1] + q[5]) + (q[3] + q[7]));
        }
        named_sync(kBarConsumers, kConsumerThreads);
        if (tid == 0) {
            s.ctl[kCtlFail] = 0;
            st_release_sys(reinterpret_cast<uint32_t *>(p.xch + kXchDFlags) + cta, token);
            const uint64_t xdl = globaltimer_ns() + p.timeout_ns;
            for (int rk = 0; rk < p.world; ++rk) {
                if (rk == p.rank) continue;
                if (!wait_flag_sys(reinterpret_cast<const uint32_t *>(p.xpeer[rk] + kXchDFlags) + cta, token, xdl)) {
                    atomicExch(&p.ctl->status, (uint32_t)MMRS_ERR_TIMEOUT);
                    atomicExch(reinterpret_cast<uint32_t *>(p.xch + kXchStatus), (uint32_t)MMRS_ERR_TIMEOUT);
                    s.ctl[kCtlFail] = 1;
                    break;
                }
            }
        }
        named_sync(kBarConsumers, kConsumerThreads);
        const bool xfail = *reinterpret_cast<volatile int *>(&s.ctl[kCtlFail]) != 0;
        for (int r = tid; r < nres && !xfail; r += kConsumerThreads) {
            const int row = dn_r0 + r;
            float v[kMaxRanks];
#pragma unroll
            for (int rk = 0; rk < kMaxRanks; ++rk)  // all loads in flight before the sum
                if (rk < p.world)
                    v[rk] = rk == p.rank ? mine[row]
                                         : ld_relaxed_sys_f32(reinterpret_cast<const float *>(p.xpeer[rk] + part_off) + row);
            float y = v[0];
#pragma unroll
            for (int rk = 1; rk < kMaxRanks; ++rk)
                if (rk < p.world) y = y + v[rk];
            if (p.residual) y = y + s.res_s[r];
            p.y[row] = y;
        }
    }
    // No copy may still be landing in shared memory when the CTA retires (after an expired wait
    // a unit may have been issued and never waited for).
    if (tid == 0 && ok1) {
        for (int st = 0; st < p.stages; ++st) {
            const int k = *reinterpret_cast<volatile int *>(&s.ticket[st]);
            if (k >= 0) mbar_wait_bounded(&s.full[st], (uint32_t)(k / p.stages) & 1u, deadline + 1000000000ull);
        }
    }
    if (tid == 0 && p.trace) p.trace[cta * 16 + 7] = globaltimer_ns();
}

// ------------------------------------------------------------------------------------------
// Host side
// ------------------------------------------------------------------------------------------
size_t decode_smem_bytes(const DecodeParams &p) {
    auto a16 = [](size_t v) { return (v + 15) / 16 * 16; };
    size_t b = a16((size_t)p.stages * p.stage_bytes) + a16(sizeof(uint64_t) * p.stages) + a16(sizeof(uint64_t));
    b += a16(p.H) + 2 * a16(4 * (p.H / 32)) + a16(16 * (p.H / 64));
    b += a16((size_t)kTopK * p.I) + 2 * a16(4 * kTopK * (p.I / 32)) + a16(16 * kTopK * (p.I / 64));
    b += a16(4 * 16) + a16(4 * 256) + a16(4 * 128) + 3 * a16(4 * kTopK);  // part, sig, cand, ids, vslot, w
    b += a16(4 * (size_t)p.res_slots * kTopK) + 2 * a16(4 * (size_t)p.act_slots) + a16(4 * (size_t)p.res_slots);
    b += a16(16 * kMaxUnits) + 2 * a16(4 * kMaxUnits) + a16(8 * kMaxUnits) + a16(4 * kMaxUnits) + a16(8 * kMaxSubs);
    b += 2 * a16(4 * (size_t)p.stages) + a16(4 * kCtlWords);
    return b;
}

static int pow2_at_least(int v) {
    int r = 1;
    while (r < v) r <<= 1;
    return r;
}

int decode_configure(DecodeParams &p, int num_sms, int max_smem) {
    if (p.H % QK_K || p.I % QK_K || p.E < kTopK || p.E > 256 || p.E % 4) return MMRS_ERR_UNSUPPORTED;
    if ((p.gu_type != MMRS_Q4K && p.gu_type != MMRS_Q5K) || (p.dn_type != MMRS_Q4K && p.dn_type != MMRS_Q5K))
        return MMRS_ERR_UNSUPPORTED;
    if (p.H / 8 / 4 > 128) return MMRS_ERR_UNSUPPORTED;  // router slice: at most 4 float4 a lane (H <= 4096)
    const int gu_tasks = (p.H / QK_K) * 4, dn_tasks = (p.I / QK_K) * 4;
    p.gu_lanes = pow2_at_least((gu_tasks + kTPL - 1) / kTPL);
    p.dn_lanes = pow2_at_least((dn_tasks + kTPL - 1) / kTPL);
    if (p.gu_lanes > 32 || p.dn_lanes > 32) return MMRS_ERR_UNSUPPORTED;  // H, I <= 6144
    // one warp's share: (32 / L) lane groups x 2 rows; a gate/up copy unit is three shares
    p.gu_sub_rows = (32 / p.gu_lanes) * kRowsPerLane;
    p.dn_sub_rows = (32 / p.dn_lanes) * kRowsPerLane;
    p.gu_unit_rows = kSubsPerGuUnit * p.gu_sub_rows;
    p.act_slots = 32 * ((kTopK * p.I / 32 + num_sms - 1) / num_sms) + 1;  // whole Q8_1 blocks a CTA
    p.res_slots = (p.H + num_sms - 1) / num_sms + 1;
    if (p.E > 2 * num_sms || num_sms > kMaxGridCtas) return MMRS_ERR_UNSUPPORTED;
    // table bounds: a CTA's gate/up chunks (one lane each; each slot boundary may add one), units
    // and sub-units
    const int max_chunks = (p.act_slots + p.gu_unit_rows - 1) / p.gu_unit_rows + kTopK;
    const int max_dn_sub = (p.res_slots + p.dn_sub_rows - 1) / p.dn_sub_rows;
    if (max_chunks > 32 || 2 * max_chunks + kTopK > kMaxUnits ||
        2 * max_chunks * kSubsPerGuUnit + kTopK * max_dn_sub > kMaxSubs || p.res_slots > 0xffff)
        return MMRS_ERR_UNSUPPORTED;
    const size_t gu_stage = kq_row_bytes(p.gu_type, p.H) * p.gu_unit_rows;
    const size_t dn_stage = kq_row_bytes(p.dn_type, p.I) * (p.res_slots - 1);
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
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
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
