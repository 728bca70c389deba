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
//   P1  the producer warp waits for barrier #1, selects the top-8 (one warp: 8 keys a lane,
//       rounds of redux max / min on order-preserving keys) and builds the copy table with its
//       32 lanes; meanwhile the consumer warps quantise x to Q8_1 and prefetch the residual.
//   P2  gate/up: the CTA owns a contiguous range of (slot, row) pairs; copy units of up to four
//       warp shares of rows of the gate or the up matrix (one bulk copy each) stream through a
//       ring of shared-memory stages.  Consumer warps claim sub-units (one warp's rows) in unit
//       order from a CTA counter, so a free warp always takes the oldest unclaimed rows; the last
//       finisher of a unit frees its stage.  The producer issues every unit as soon as its stage
//       is free, so the down units (this CTA's output rows of one expert: one contiguous copy
//       each) land in the ring while gate/up is still being computed.
//   P3  act = up * silu(gate) of the CTA's range goes to global memory as f32; grid barrier #2;
//       every CTA reads the whole act vector back (one 16-byte load per lane and 128 values, all
//       of a warp's loads in flight together) and quantises it to Q8_1 itself
//       (quantize_silu_mul_q8_1 arithmetic, no cross-CTA hand-off); then the down sub-units,
//       weighted by the route weight, the reference's fixed 8-way tree
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
constexpr int kSubsPerGuUnit = 4;
constexpr int kMaxUnits = 80;
constexpr int kMaxSubs = 256;
constexpr int kTopK = 8;
constexpr int kTPL = 3;  // tasks (64-weight sub-block pairs) per lane
constexpr int kRouterRounds = (16 + kWarps - 1) / kWarps;
// named barriers: consumers, table ready (all threads), router partials (all threads)
constexpr int kBarConsumers = 1, kBarTable = 3, kBarRouter = 4;
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

// 128 consecutive values, lane l holding values 4l..4l+3 (Q8_1 blocks of 32 over 8 lanes):
// d = amax/127, q = roundf(v/d) (quantize_q8_1, gguf.cuh:1234-1261, and quantize_silu_mul_q8_1,
// moe_gguf.cu:255-284).  Writes q, and per block the fp16-rounded scale d and the sum of quants S.
__device__ __forceinline__ void quant128(float4 v, int8_t *q, float *d, int *S, int lane) {
    float amax = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
#pragma unroll
    for (int m = 4; m > 0; m >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, m));
    const float dd = __fdiv_rn(amax, 127.0f);
    int q0 = 0, q1 = 0, q2 = 0, q3 = 0;
    if (amax != 0.f) {
        q0 = (int)roundf(__fdiv_rn(v.x, dd));
        q1 = (int)roundf(__fdiv_rn(v.y, dd));
        q2 = (int)roundf(__fdiv_rn(v.z, dd));
        q3 = (int)roundf(__fdiv_rn(v.w, dd));
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
    uint64_t *full, *empty;
    int8_t *xq;                // [H]
    float *xd;                 // [H/32]
    int *xS;                   // [H/32]
    float4 *xts;               // [H/64]
    int8_t *aq_s;              // [8][I] (positions)
    float *ad_s;               // [8][I/32]
    int *aS_s;                 // [8][I/32]
    float4 *ats;               // [8][I/64]
    float *part;               // router slice sums [2][8]
    int *ids;                  // [8] expert of each slot (-1: none, or another rank's)
    int *vslot;                // [8] slot of each position (the computed slots in order)
    float *w;                  // [8]
    float *dn_acc;             // [res_slots][8] weighted expert rows of this CTA's output range
    float *gval, *uval;        // [act_slots] gate / up row values of this CTA's (position, row) range
    float *res_s;              // [res_slots]
    int4 *units;               // [kMaxUnits]
    int *unit_off;             // [kMaxUnits] first row of a gate/up unit in the CTA's range
    int *unit_nsub;            // [kMaxUnits] sub-units of the unit
    int2 *subs;                // [kMaxSubs]
    int *ticket;               // [stages] unit last issued into each stage
    int *done;                 // [stages] sub-units of the stage's unit finished
    int *ctl;                  // [kCtlWords]
};

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
        s.empty = reinterpret_cast<uint64_t *>(take(sizeof(uint64_t) * p.stages));
        s.xq = reinterpret_cast<int8_t *>(take(H));
        s.xd = reinterpret_cast<float *>(take(sizeof(float) * (H / 32)));
        s.xS = reinterpret_cast<int *>(take(sizeof(int) * (H / 32)));
        s.xts = reinterpret_cast<float4 *>(take(sizeof(float4) * (H / 64)));
        s.aq_s = reinterpret_cast<int8_t *>(take((size_t)kTopK * I));
        s.ad_s = reinterpret_cast<float *>(take(sizeof(float) * kTopK * (I / 32)));
        s.aS_s = reinterpret_cast<int *>(take(sizeof(int) * kTopK * (I / 32)));
        s.ats = reinterpret_cast<float4 *>(take(sizeof(float4) * kTopK * (I / 64)));
        s.part = reinterpret_cast<float *>(take(sizeof(float) * 16));
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
            mbar_init(&s.empty[i], 1);
            s.ticket[i] = -1;
            s.done[i] = 0;
        }
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
        // ---- routing: lane l holds experts l + 32 i ------------------------------------------
        int slot_id = -1;  // lane k < 8: expert of slot k
        float slot_w = 0.f;
        if (p.internal_routing) {
            if (ok) {
                uint32_t key[8];
                float sg[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int e = lane + 32 * i;
                    key[i] = 0u;  // experts >= E are never selected (E >= 8 real keys are > 0)
                    sg[i] = 0.f;
                    if (e < E) {
                        const float l = __ldcg(p.logits + e);
                        sg[i] = __fdiv_rn(1.0f, 1.0f + expf(-l));
                        key[i] = sel_key(sg[i], __ldg(p.bias + e));
                    }
                }
                // stable descending order of the score: larger key first, lower expert id on ties
                uint32_t taken = 0u;
                float my_sig = 0.f;
#pragma unroll
                for (int k = 0; k < kTopK; ++k) {
                    uint32_t bk = 0u;
                    int bi = 0;
                    float bs = 0.f;
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        if (!(taken & (1u << i)) && key[i] > bk) {
                            bk = key[i];
                            bi = i;
                            bs = sg[i];
                        }
                    const uint32_t mk = __reduce_max_sync(0xffffffffu, bk);
                    const uint32_t mine = (uint32_t)(lane + 32 * bi);
                    const uint32_t me = __reduce_min_sync(0xffffffffu, bk == mk ? mine : 0xffffffffu);
                    if (mine == me) taken |= 1u << bi;
                    const float sme = __shfl_sync(0xffffffffu, bs, (int)(me & 31u));
                    if (lane == k) {
                        slot_id = (int)me;
                        my_sig = sme;
                    }
                }
                // weights: sig / ((v0+v4)+(v2+v6))+((v1+v5)+(v3+v7)), lane k keeps w_k
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
        // ---- copy table: lane c computes gate/up chunk c of the CTA's (position, row) range --
        const int gu_p0 = (int)((int64_t)cta * nvs * I / G), gu_p1 = (int)((int64_t)(cta + 1) * nvs * I / G);
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
        // ---- issue loop (lane 0) ----------------------------------------------------------------
        if (lane == 0 && ok) {
            const int n = n_gu_units + n_dn_units;
            int k = 0;
            for (; k < n; ++k) {
                const int st = k % p.stages;
                if (!mbar_wait_sleep(&s.empty[st], ((uint32_t)(k / p.stages) & 1u) ^ 1u, deadline)) {
                    atomicExch(&p.ctl->status, (uint32_t)MMRS_ERR_TIMEOUT);
                    break;
                }
                *reinterpret_cast<volatile int *>(&s.ticket[st]) = k;
                const int4 u = s.units[k];
                const int e = s.ids[s.vslot[u.y]];
                const uint8_t *src;
                uint32_t bytes;
                if (u.x == 2) {
                    src = p.down + (size_t)e * dn_expert_bytes + (size_t)u.z * dn_row_bytes;
                    bytes = (uint32_t)(dn_row_bytes * u.w);
                } else {
                    src = (u.x == 0 ? p.gate : p.up) + (size_t)e * gu_expert_bytes + (size_t)u.z * gu_row_bytes;
                    bytes = (uint32_t)(gu_row_bytes * u.w);
                }
                if (k == 0 && p.trace) p.trace[cta * 16 + 8] = globaltimer_ns();
                if (k == n_gu_units && p.trace) p.trace[cta * 16 + 10] = globaltimer_ns();
                mbar_arrive_expect_tx_sink(&s.full[st], bytes);
                bulk_g2s(s.stages + (size_t)st * p.stage_bytes, src, bytes, &s.full[st]);
            }
            if (p.trace) p.trace[cta * 16 + 9] = globaltimer_ns();
            // Drain: no copy may still be landing in shared memory when the CTA retires.
            const int first = k > p.stages ? k - p.stages : 0;
            for (int j = first; j < k; ++j)
                mbar_wait_bounded(&s.full[j % p.stages], (uint32_t)(j / p.stages) & 1u, deadline + 1000000000ull);
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
    named_sync(kBarTable, kThreads);
    const bool ok1 = s.ctl[kCtlOk] != 0;
    const int n_sub_gu = s.ctl[kCtlSubGu], n_sub = s.ctl[kCtlSubs], nvs = s.ctl[kCtlPositions];
    bool aborted = !ok1;
    auto claim = [&]() -> int {
        int v = 0;
        if (lane == 0) v = atomicAdd(&s.ctl[kCtlNext], 1);
        return __shfl_sync(0xffffffffu, v, 0);
    };
    // A warp that finished a sub-unit of unit k: the last finisher frees the unit's stage.
    auto finish = [&](int k, int st) {
        __syncwarp();
        if (lane == 0) {
            const int old = atom_add_acq_rel_cta(&s.done[st], 1);
            if (old + 1 == s.unit_nsub[k]) {
                s.done[st] = 0;
                mbar_arrive(&s.empty[st]);
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
                if (p.gu_type == MMRS_Q5K) {
                    vA = row_dot<MMRS_Q5K>(rowA, lig, Lg, ntasks, ta);
                    vB = row_dot<MMRS_Q5K>(rowB, lig, Lg, ntasks, ta);
                } else {
                    vA = row_dot<MMRS_Q4K>(rowA, lig, Lg, ntasks, ta);
                    vB = row_dot<MMRS_Q4K>(rowB, lig, Lg, ntasks, ta);
                }
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

    // ---- P3: act of the CTA's range to global memory, grid barrier #2 -------------------------
    named_sync(kBarConsumers, kConsumerThreads);  // every gate/up sub-unit of this CTA is done
    if (tid == 0 && p.trace) p.trace[cta * 16 + 4] = globaltimer_ns();
    {
        const int gu_p0 = (int)((int64_t)cta * nvs * I / G), gu_p1 = (int)((int64_t)(cta + 1) * nvs * I / G);
        for (int i = tid; i < gu_p1 - gu_p0; i += kConsumerThreads) {
            const float gv = s.gval[i];
            // act = up * silu(gate) (moe_gguf.cu:272-273)
            p.act[gu_p0 + i] = aborted ? 0.f : s.uval[i] * __fdiv_rn(gv, 1.0f + expf(-gv));
        }
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
        s.ctl[kCtlFail] = ok2 ? 0 : 1;
        if (ok2) p.ctl->epoch[cta] = epoch + 2u;  // read again only by this CTA's next launch
        if (p.trace) p.trace[cta * 16 + 5] = globaltimer_ns();
    }
    named_sync(kBarConsumers, kConsumerThreads);
    if (s.ctl[kCtlFail]) aborted = true;
    // Every CTA quantises the whole act vector: 128 values per warp step (one float4 a lane),
    // all of a warp's loads in flight before its first block is quantised.
    {
        const int nchunk = nvs * I / 128;
        constexpr int kLd = 8;
        for (int c0 = warp * kLd; c0 < nchunk; c0 += kConsumerWarps * kLd) {
            float4 v[kLd];
#pragma unroll
            for (int j = 0; j < kLd; ++j)
                v[j] = (c0 + j < nchunk && !aborted) ? __ldcg(reinterpret_cast<const float4 *>(p.act) + (c0 + j) * 32 + lane)
                                                     : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int j = 0; j < kLd; ++j) {
                const int c = c0 + j;
                if (c < nchunk) quant128(v[j], s.aq_s + c * 128, s.ad_s + c * 4, s.aS_s + c * 4, lane);
            }
        }
        named_sync(kBarConsumers, kConsumerThreads);
        build_task_scales(s.ats, s.ad_s, s.aS_s, nvs * (I / 64), tid, kConsumerThreads);
        named_sync(kBarConsumers, kConsumerThreads);
        if (tid == 0 && p.trace) p.trace[cta * 16 + 6] = globaltimer_ns();
    }

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
                if (p.dn_type == MMRS_Q5K) {
                    vA = row_dot<MMRS_Q5K>(rowA, lig, Ld, ntasks, ta);
                    vB = row_dot<MMRS_Q5K>(rowB, lig, Ld, ntasks, ta);
                } else {
                    vA = row_dot<MMRS_Q4K>(rowA, lig, Ld, ntasks, ta);
                    vB = row_dot<MMRS_Q4K>(rowB, lig, Ld, ntasks, ta);
                }
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
    if (tid == 0 && p.trace) p.trace[cta * 16 + 7] = globaltimer_ns();
}

// ------------------------------------------------------------------------------------------
// Host side
// ------------------------------------------------------------------------------------------
size_t decode_smem_bytes(const DecodeParams &p) {
    auto a16 = [](size_t v) { return (v + 15) / 16 * 16; };
    size_t b = a16((size_t)p.stages * p.stage_bytes) + 2 * a16(sizeof(uint64_t) * p.stages);
    b += a16(p.H) + 2 * a16(4 * (p.H / 32)) + a16(16 * (p.H / 64));
    b += a16((size_t)kTopK * p.I) + 2 * a16(4 * kTopK * (p.I / 32)) + a16(16 * kTopK * (p.I / 64));
    b += a16(4 * 16) + 3 * a16(4 * kTopK);  // part, ids, vslot, w
    b += a16(4 * (size_t)p.res_slots * kTopK) + 2 * a16(4 * (size_t)p.act_slots) + a16(4 * (size_t)p.res_slots);
    b += a16(16 * kMaxUnits) + 2 * a16(4 * kMaxUnits) + a16(8 * kMaxSubs);
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
    // one warp's share: (32 / L) lane groups x 2 rows; a gate/up copy unit is four shares
    p.gu_sub_rows = (32 / p.gu_lanes) * kRowsPerLane;
    p.dn_sub_rows = (32 / p.dn_lanes) * kRowsPerLane;
    p.gu_unit_rows = kSubsPerGuUnit * p.gu_sub_rows;
    p.act_slots = (kTopK * p.I + num_sms - 1) / num_sms + 1;
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

int decode_launch(const DecodeParams &p, cudaStream_t stream) {
    const size_t smem = decode_smem_bytes(p);
    // Raise the dynamic shared-memory limit once per device (the attribute is per context);
    // call_once keeps concurrent host threads from racing on it.
    static std::once_flag once[64];
    static cudaError_t set_rc[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return MMRS_ERR_LAUNCH;
    std::call_once(once[dev], [dev] {
        int optin = 0;
        cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        set_rc[dev] = cudaFuncSetAttribute(moe_decode_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, optin);
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
    const cudaError_t err = cudaLaunchKernelEx(&cfg, moe_decode_fused_kernel, p);
    return err == cudaSuccess ? MMRS_OK : MMRS_ERR_LAUNCH;
}

}  // namespace mmrs
