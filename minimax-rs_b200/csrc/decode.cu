// Fused single-token MoE block for B200 (sm_100a).
//
// Replaces, in one persistent launch, the reference's decode chain
//   router Linear (fused_moe.rs:267) -> minimax_moe_decode_topk (moe_gguf.cu:34-100)
//   -> quantize_q8_1 -> moe_gate_up_decode_kernel -> quantize_silu_mul_q8_1
//   -> moe_down_decode_kernel (moe_gguf.cu:200-343, 426-567) -> + residual (model.rs:218)
//
// One CTA per SM: 12 consumer warps (three groups of 4) + 1 producer warp.
//   P0  router GEMV in the canonical order (8 K-slices; the CTA's two experts x 8 slices are 16
//       (expert, slice) pairs, pair w + 12 r to consumer warp w: 32 lane partials, butterfly,
//       fixed slice tree); every CTA quantises x to Q8_1 in shared memory.  Grid barrier #1.
//   P1  every CTA selects the top-8 with warp-shuffle argmax rounds on 64-bit keys
//       (score desc, expert id asc — the stable descending order) and renormalises the weights
//       with the reference's fixed tree.
//   P2  gate/up: each CTA owns a contiguous range of (slot, row) pairs, streamed in units of up
//       to 8 rows x {gate, up} into a ring of shared-memory stages by 1-D bulk TMA copies
//       (cp.async.bulk + mbarrier complete_tx).  Consumer groups take alternate units; in a group
//       a half-warp computes one gate row, the other half the matching up row, and
//       act = up * silu(gate) stays in shared memory.  Q8_1 blocks of act inside the CTA's range
//       are quantised locally; a block shared with a neighbour CTA goes through global scratch
//       and is quantised by whichever CTA completes it.
//   P3  grid barrier #2, one bulk copy of the quantised activation per CTA; down: each CTA owns a
//       contiguous range of output rows, units of rows x 8 routed experts (the producer streams
//       them during P2 already); the 8 expert values of a row are summed with the reference's
//       tree ((v0+v4)+(v2+v6))+((v1+v5)+(v3+v7)) and the residual is added.
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

constexpr int kGroupWarps = 4;
// 3 groups of 4 consumer warps + the producer = 13 warps (at most 4 on a scheduler): 128 registers
// a thread; 4 groups (17 warps, 5 on one scheduler) capped the kernel at 96 with spills.
constexpr int kGroups = 3;
constexpr int kRowsPerLane = 2;   // rows a lane group computes per unit (same activation registers)
constexpr int kMaxUnits = 96;
constexpr int kConsumerWarps = kGroupWarps * kGroups;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kRouterRounds = (16 + kConsumerWarps - 1) / kConsumerWarps;  // 2 experts x 8 K-slices per CTA
constexpr int kThreads = kConsumerThreads + 32;
constexpr int kTopK = 8;
constexpr int kTPL = 3;  // tasks (64-weight sub-block pairs) per lane

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
// d = amax/127, q = roundf(v/d) (quantize_q8_1, gguf.cuh:1234-1261).  Writes q, and per block the
// fp16-rounded scale d and the sum of quants S.
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

// Consumer wait for unit k in stage st: first the stage's ticket (the producer has issued unit k
// there), then the phase of the full barrier.  Bounded by the deadline.
__device__ __forceinline__ bool wait_unit(uint64_t *full, const int *ticket, int k, int st, int stages,
                                          uint64_t deadline) {
    uint32_t spins = 0;
    while (*reinterpret_cast<const volatile int *>(&ticket[st]) != k) {
        __nanosleep(64);
        if ((++spins & 255u) == 0 && globaltimer_ns() > deadline) return false;
    }
    // sleeping wait: a group waiting for its data leaves the issue slots to the groups computing
    return mbar_wait_sleep(&full[st], (uint32_t)(k / stages) & 1u, deadline);
}

// Unit enumeration shared by producer and consumers (identical sequences).
struct GuUnit {
    int slot, row0, n;
};
__device__ __forceinline__ GuUnit gu_unit_at(int p, int pend, int I, int U) {
    GuUnit u;
    u.slot = p / I;
    u.row0 = p - u.slot * I;
    const int a = pend - p, b = I - u.row0;
    u.n = min(U, min(a, b));
    return u;
}

struct DecodeSmem {
    uint8_t *stages;
    uint64_t *full, *empty, *abar;
    int8_t *xq;                // [H]
    float *xd;                 // [H/32]
    int *xS;                   // [H/32]
    float4 *xts;               // [H/64]
    int8_t *aq_s;              // [8][I]
    float *ad_s;               // [8][I/32]
    int *aS_s;                 // [8][I/32]
    float4 *ats;               // [8][I/64]
    float *part;               // router slice sums [2][8] in P0, selection scores [E] in P1
    float *sig;                // [E]
    int *ids;                  // [8]
    int *vslot;                // [8] slots in gate/up position order (valid first under EP)
    int *vpos;                 // [8] position block of each slot in act / aq
    float *w;                  // [8]
    float *dn_acc;             // [res_slots][8]
    float *act_s;              // [act_slots]
    float *gval, *uval;        // [act_slots] gate / up row values of this CTA's range
    int4 *units;               // [kMaxUnits] (kind, slot, first row, rows)
    int *unit_off;             // [kMaxUnits] offset of the first row in the CTA's range
    int *ticket;               // [stages] index of the unit last issued into each stage
    int *n_gu;
    float *res_s;              // [res_slots]
    uint32_t *base;
    int *flag;
};

__global__ void __launch_bounds__(kThreads, 1) moe_decode_fused_kernel(const __grid_constant__ DecodeParams p) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, cta = blockIdx.x;
    const int H = p.H, I = p.I, E = p.E;
    const uint64_t t_start = globaltimer_ns();
    const uint64_t deadline = t_start + p.timeout_ns;
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
        s.abar = reinterpret_cast<uint64_t *>(take(sizeof(uint64_t)));
        s.xq = reinterpret_cast<int8_t *>(take(H));
        s.xd = reinterpret_cast<float *>(take(sizeof(float) * (H / 32)));
        s.xS = reinterpret_cast<int *>(take(sizeof(int) * (H / 32)));
        s.xts = reinterpret_cast<float4 *>(take(sizeof(float4) * (H / 64)));
        s.aq_s = reinterpret_cast<int8_t *>(take((size_t)kTopK * I));
        s.ad_s = reinterpret_cast<float *>(take(sizeof(float) * kTopK * (I / 32)));
        s.aS_s = reinterpret_cast<int *>(take(sizeof(int) * kTopK * (I / 32)));
        s.ats = reinterpret_cast<float4 *>(take(sizeof(float4) * kTopK * (I / 64)));
        s.part = reinterpret_cast<float *>(take(sizeof(float) * (E > 16 ? E : 16)));
        s.sig = reinterpret_cast<float *>(take(sizeof(float) * E));
        s.ids = reinterpret_cast<int *>(take(sizeof(int) * kTopK));
        s.vslot = reinterpret_cast<int *>(take(sizeof(int) * kTopK));
        s.vpos = reinterpret_cast<int *>(take(sizeof(int) * kTopK));
        s.w = reinterpret_cast<float *>(take(sizeof(float) * kTopK));
        s.dn_acc = reinterpret_cast<float *>(take(sizeof(float) * p.res_slots * kTopK));
        s.act_s = reinterpret_cast<float *>(take(sizeof(float) * p.act_slots));
        s.gval = reinterpret_cast<float *>(take(sizeof(float) * p.act_slots));
        s.uval = reinterpret_cast<float *>(take(sizeof(float) * p.act_slots));
        s.units = reinterpret_cast<int4 *>(take(sizeof(int4) * kMaxUnits));
        s.unit_off = reinterpret_cast<int *>(take(sizeof(int) * kMaxUnits));
        s.ticket = reinterpret_cast<int *>(take(sizeof(int) * p.stages));
        s.n_gu = reinterpret_cast<int *>(take(16));
        s.res_s = reinterpret_cast<float *>(take(sizeof(float) * p.res_slots));
        s.base = reinterpret_cast<uint32_t *>(take(16));
        s.flag = reinterpret_cast<int *>(take(16));
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
            mbar_init(&s.empty[i], kGroupWarps);
            s.ticket[i] = -1;
        }
        mbar_init(s.abar, 1);
        fence_mbar_init();
        s.flag[0] = 1;
        s.flag[1] = 0;
    }
    __syncthreads();

    const int dn_r0 = (int)((int64_t)cta * H / G), dn_r1 = (int)((int64_t)(cta + 1) * H / G);
    const size_t gu_row_bytes = kq_row_bytes(p.gu_type, H);
    const size_t dn_row_bytes = kq_row_bytes(p.dn_type, I);
    const size_t gu_expert_bytes = gu_row_bytes * I;
    const size_t dn_expert_bytes = dn_row_bytes * H;

    // ---- P0: router slices, Q8_1 of x, residual prefetch (all loads issued before use) ----
    if (warp < kConsumerWarps) {
        const int nxc = H / 128;  // chunks of 128 values
        float4 xv[2];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int c = warp + kConsumerWarps * i;
            if (c < nxc) xv[i] = __ldg(reinterpret_cast<const float4 *>(p.x) + c * 32 + lane);
        }
        float rv = 0.f;
        const int rrow = dn_r0 + tid;
        if (p.residual && rrow < dn_r1) rv = __ldg(p.residual + rrow);
        // router pairs (expert le of this CTA's two, K-slice sl): pair pi = warp + kConsumerWarps * r
        const int slice = H / 8, groups = slice / 4;
        float4 xx[kRouterRounds][4], wv[kRouterRounds][4];
#pragma unroll
        for (int r = 0; r < kRouterRounds; ++r) {
            const int pi = warp + kConsumerWarps * r, sl = pi & 7, le = pi >> 3;
            const int e = cta + G * le;
            if (pi < 16 && p.internal_routing && e < E) {
                const float4 *xs = reinterpret_cast<const float4 *>(p.x + sl * slice);
                const float4 *wr = reinterpret_cast<const float4 *>(p.router + (size_t)e * H + sl * slice);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int g = lane + 32 * i;
                    if (g < groups) {
                        xx[r][i] = __ldg(xs + g);
                        wv[r][i] = __ldg(wr + g);
                    }
                }
            }
        }
        // Per-block arrival counters are zeroed here: nothing increments them before barrier #1.
        for (int b = cta * kConsumerThreads + tid; b < kTopK * (I / 32); b += G * kConsumerThreads)
            p.blk_count[b] = 0u;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int c = warp + kConsumerWarps * i;
            if (c < nxc) quant128(xv[i], s.xq + c * 128, s.xd + c * 4, s.xS + c * 4, lane);
        }
        if (p.residual && rrow < dn_r1) s.res_s[tid] = rv;
#pragma unroll
        for (int r = 0; r < kRouterRounds; ++r) {
            const int pi = warp + kConsumerWarps * r, sl = pi & 7, le = pi >> 3;
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
        if (tid == 0) s.base[0] = __ldcg(&p.ctl->epoch[cta]);
        named_sync(1, kConsumerThreads);
        build_task_scales(s.xts, s.xd, s.xS, H / 64, tid, kConsumerThreads);
        if (p.internal_routing && tid < 2) {
            const int ee = cta + G * tid;
            if (ee < E) {
                const float *q = s.part + tid * 8;
                p.logits[ee] = ((q[0] + q[1]) + (q[2] + q[3])) + ((q[4] + q[5]) + (q[6] + q[7]));
            }
        }
    }
    if (tid == 0 && p.trace) p.trace[cta * 16 + 1] = globaltimer_ns();

    // ---- P1: routing ----------------------------------------------------------------------
    __syncthreads();
    const uint32_t epoch = s.base[0];
    bool ok = grid_sync(p.ctl, (uint32_t)G * (epoch + 1u), deadline, s.flag, 2, kThreads);
    if (tid == 0 && p.trace) p.trace[cta * 16 + 2] = globaltimer_ns();
    if (p.internal_routing) {
        if (ok) {
            // Selection score sigmoid(l) + bias as an order-preserving 32-bit key (-0 as +0); the
            // stable descending order is "larger key first, lower expert id on equal keys".
            // Warp w holds experts [32 w, 32 w + 32) and extracts its top 8 by rounds of redux max
            // (key) and redux min (id among the lanes holding that key); warp 0 merges the
            // candidates the same way.  Candidates (key, id) reuse the score array.
            const int nw = (E + 31) / 32;
            uint32_t *cand = reinterpret_cast<uint32_t *>(s.part);  // [2][8 nw] <= max(E, 16) words
            if (warp < nw) {
                const int e = tid;
                uint32_t key = 0u;  // experts >= E: never selected (E >= 8 real keys are > 0)
                if (e < E) {
                    const float l = __ldcg(p.logits + e);
                    const float sg = __fdiv_rn(1.0f, 1.0f + expf(-l));
                    s.sig[e] = sg;
                    float sv = sg + p.bias[e];
                    if (sv == 0.0f) sv = 0.0f;
                    const uint32_t u = __float_as_uint(sv);
                    key = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
                }
                bool taken = false;
#pragma unroll
                for (int k = 0; k < kTopK; ++k) {
                    const uint32_t mk = __reduce_max_sync(0xffffffffu, taken ? 0u : key);
                    const uint32_t me =
                        __reduce_min_sync(0xffffffffu, (!taken && key == mk) ? (uint32_t)e : 0xffffffffu);
                    taken |= (uint32_t)e == me;
                    if (lane == 0) {
                        cand[warp * kTopK + k] = mk;
                        cand[8 * nw + warp * kTopK + k] = me;
                    }
                }
            }
            __syncthreads();
            if (warp == 0) {
                const int nc = 8 * nw;
                const uint32_t ka = lane < nc ? cand[lane] : 0u, ia = lane < nc ? cand[nc + lane] : 0xffffffffu;
                const uint32_t kb = lane + 32 < nc ? cand[lane + 32] : 0u;
                const uint32_t ib = lane + 32 < nc ? cand[nc + lane + 32] : 0xffffffffu;
                bool ta = false, tb = false;
                int myid = 0;
#pragma unroll
                for (int k = 0; k < kTopK; ++k) {
                    const uint32_t mk = __reduce_max_sync(0xffffffffu, max(ta ? 0u : ka, tb ? 0u : kb));
                    const uint32_t ca = (!ta && ka == mk) ? ia : 0xffffffffu;
                    const uint32_t cb = (!tb && kb == mk) ? ib : 0xffffffffu;
                    const uint32_t me = __reduce_min_sync(0xffffffffu, min(ca, cb));
                    if (ca == me) ta = true;
                    else if (cb == me) tb = true;
                    if (lane == k) myid = (int)me;
                }
                // weights: sig / ((v0+v4)+(v2+v6))+((v1+v5)+(v3+v7)) on every lane, lane k keeps w_k
                const float vk = lane < kTopK ? s.sig[myid] : 0.0f;
                float v[kTopK];
#pragma unroll
                for (int k = 0; k < kTopK; ++k) v[k] = __shfl_sync(0xffffffffu, vk, k);
                const float denom = ((v[0] + v[4]) + (v[2] + v[6])) + ((v[1] + v[5]) + (v[3] + v[7]));
                if (lane < kTopK) {
                    const float wk = __fdiv_rn(vk, denom);
                    s.ids[lane] = myid;
                    s.w[lane] = wk;
                    if (cta == 0) {
                        if (p.topk_ids_out) p.topk_ids_out[lane] = (uint32_t)myid;
                        if (p.topk_w_out) p.topk_w_out[lane] = wk;
                    }
                }
            }
        }
    } else {
        if (tid < kTopK) {
            s.ids[tid] = -1;
            s.w[tid] = 0.f;
        }
        __syncthreads();
        if (tid < kTopK) {
            // (route, expert) pairs in expert order; routes outside [0, 8) and invalid experts
            // contribute nothing, as in moe_down_decode_kernel (moe_gguf.cu:311)
            const int slot = p.ext_route[tid];
            const int e = p.ext_expert[tid];
            if (slot >= 0 && slot < kTopK) {
                s.ids[slot] = (e >= 0 && e < E) ? e : -1;
                s.w[slot] = p.ext_w[slot];
            }
        }
    }
    // Gate/up position space: the (slot, row) pairs of the computed experts, partitioned evenly
    // over the CTAs.  Single GPU and TP: all 8 slots in order.  Expert parallel: experts owned by
    // other ranks contribute nothing here and their slots are left out, so this rank's CTAs share
    // only its own experts' rows.  Warp 0 (whose lanes 0..7 wrote ids in both routing paths).
    const bool compact = p.world > 1 && p.ep;
    if (warp == 0) {
        __syncwarp();
        int id = lane < kTopK ? s.ids[lane] : -1;
        if (compact && id >= 0 && id % p.world != p.rank) id = -1;
        const bool keep = lane < kTopK && (!compact || id >= 0);
        const uint32_t kept = __ballot_sync(0xffffffffu, keep);
        const int nv = __popc(kept);
        if (lane < kTopK) {
            const uint32_t below = (1u << lane) - 1u;
            const int pos = keep ? __popc(kept & below) : nv + __popc(~kept & 0xFFu & below);
            s.ids[lane] = id;
            s.vslot[pos] = lane;
            s.vpos[lane] = pos;
        }
        if (lane == 0) s.n_gu[2] = nv;
    }
    __syncthreads();
    const int nvs = s.n_gu[2];
    const int gu_p0 = (int)((int64_t)cta * nvs * I / G), gu_p1 = (int)((int64_t)(cta + 1) * nvs * I / G);
    if (!ok) return;  // nothing issued yet
    if (tid == 0 && p.trace) p.trace[cta * 16 + 3] = globaltimer_ns();

    // Unit table.  Every unit is ONE contiguous bulk copy (few, large TMA operations keep the
    // per-SM copy engine at HBM rate): a chunk of up to U_gu rows of the gate or of the up matrix
    // of one routed expert (gate chunk, then the matching up chunk), then one down unit per routed
    // expert covering this CTA's output rows (split every U_dn rows).  Unit k goes to ring stage
    // k % stages and to consumer group k % kGroups.  Entry: (kind 0 gate / 1 up / 2 down, slot,
    // first row, rows); for gate/up the offset of the first row in the CTA's (slot,row) range is
    // row-offset field .w >> 8 ... stored separately in gu_off.
    const int U_gu = p.gu_unit_rows, U_dn = p.dn_unit_rows;
    if (warp == kConsumerWarps) {
        // ---------------------------- producer --------------------------------------------
        // Lane 0 builds the unit table and releases the consumers (named barrier 3) before it
        // issues the first copy: an issue can block on the copy engine, the consumers must not.
        int n = 0, k = 0;
        bool live = true;
        int n_gu = 0x7fffffff;  // no "first down unit" stamp while the table grows
        auto unit_src = [&](int k, uint32_t &bytes) -> const uint8_t * {
            const int4 u = s.units[k];
            const int e = s.ids[u.y];
            if (e < 0) return nullptr;
            if (u.x < 2) {
                bytes = (uint32_t)(gu_row_bytes * u.w);
                return (u.x == 0 ? p.gate : p.up) + (size_t)e * gu_expert_bytes + (size_t)u.z * gu_row_bytes;
            }
            bytes = (uint32_t)(dn_row_bytes * u.w);
            return p.down + (size_t)e * dn_expert_bytes + (size_t)u.z * dn_row_bytes;
        };
        // issue unit k into ring stage k % stages; false when the stage wait expired
        auto issue = [&](int k) -> bool {
            const int st = k % p.stages;
            if (!mbar_wait_sleep(&s.empty[st], ((uint32_t)(k / p.stages) & 1u) ^ 1u, deadline)) {
                atomicExch(&p.ctl->status, (uint32_t)MMRS_ERR_TIMEOUT);
                return false;
            }
            if (k == 0 && p.trace) p.trace[cta * 16 + 8] = globaltimer_ns();
            if (k == n_gu && p.trace) p.trace[cta * 16 + 10] = globaltimer_ns();
            // Publish which unit this stage now holds.  Consumer groups take interleaved units,
            // so a group can reach unit k before unit k - stages (another group's) has landed;
            // waiting for the ticket first keeps the parity wait from aliasing onto that phase.
            *reinterpret_cast<volatile int *>(&s.ticket[st]) = k;
            const int4 u = s.units[k];
            uint8_t *dst = s.stages + (size_t)st * p.stage_bytes;
            if (u.x == 2) {
                // rows [u.z, u.z + u.w) of all routed experts, expert q at dst + q * U_dn rows
                const uint32_t bytes = (uint32_t)(dn_row_bytes * u.w);
                uint32_t tx = 0;
                for (int q = 0; q < kTopK; ++q) tx += s.ids[q] >= 0 ? bytes : 0;
                mbar_arrive_expect_tx(&s.full[st], tx);
                for (int q = 0; q < kTopK; ++q) {
                    const int e = s.ids[q];
                    if (e < 0) continue;
                    bulk_g2s(dst + (size_t)q * dn_row_bytes * U_dn,
                             p.down + (size_t)e * dn_expert_bytes + (size_t)u.z * dn_row_bytes, bytes, &s.full[st]);
                }
                return true;
            }
            uint32_t bytes = 0;
            const uint8_t *src = unit_src(k, bytes);
            if (!src) {
                mbar_arrive(&s.full[st]);
                return true;
            }
            mbar_arrive_expect_tx(&s.full[st], bytes);
            bulk_g2s(dst, src, bytes, &s.full[st]);
            return true;
        };
        if (lane == 0) {
            // the table (each entry is written before its unit is issued)
            for (int q = gu_p0; q < gu_p1 && n + 2 <= kMaxUnits;) {
                const GuUnit u = gu_unit_at(q, gu_p1, I, U_gu);
                const int slot = s.vslot[u.slot];
                s.units[n] = make_int4(0, slot, u.row0, u.n);
                s.unit_off[n++] = q - gu_p0;
                s.units[n] = make_int4(1, slot, u.row0, u.n);
                s.unit_off[n++] = q - gu_p0;
                q += u.n;
            }
            s.n_gu[0] = n;
            for (int r = dn_r0; r < dn_r1 && n < kMaxUnits; r += U_dn) {
                s.units[n] = make_int4(2, 0, r, min(U_dn, dn_r1 - r));
                s.unit_off[n++] = r - dn_r0;
            }
            s.n_gu[1] = n;
        }
        __threadfence_block();
        __syncwarp();
        named_arrive(3, kThreads);  // the table is complete
        if (lane == 0) {
            n_gu = s.n_gu[0];
            for (; live && k < n; ++k) live = issue(k);
            if (p.trace) p.trace[cta * 16 + 9] = globaltimer_ns();
            // Drain: no copy may still be landing in shared memory when the CTA retires.
            const int first = k > p.stages ? k - p.stages : 0;
            for (int j = first; j < k; ++j)
                mbar_wait_bounded(&s.full[j % p.stages], (uint32_t)(j / p.stages) & 1u, deadline + 1000000000ull);
        }
        return;
    }
    named_sync(3, kThreads);
    const int n_gu = s.n_gu[0];
    const int n_units = s.n_gu[1];

    // ------------------------------- consumers ----------------------------------------------
    const int grp = warp / kGroupWarps, gw = warp % kGroupWarps;
    bool aborted = false;
    {
        // P2: gate / up chunks.  A lane group of L lanes computes two rows of the chunk against the
        // register-resident Q8_1 x (6 independent 64-weight task dots per lane).
        const int L = p.gu_lanes;
        const int lgi = gw * (32 / L) + lane / L, lig = lane % L;
        const int rA = lgi * kRowsPerLane, rB = rA + 1;
        const int ntasks = (H / QK_K) * 4;
        TaskAct ta[kTPL];
        load_task_acts(ActView{s.xq, s.xts}, lig, L, ntasks, ta);
        for (int k = grp; k < n_gu; k += kGroups) {
            const int4 u = s.units[k];
            const int st = k % p.stages;
            if (!aborted && !wait_unit(s.full, s.ticket, k, st, p.stages, deadline)) {
                atomicExch(&p.ctl->status, (uint32_t)MMRS_ERR_TIMEOUT);
                aborted = true;
            }
            float vA = 0.f, vB = 0.f;
            if (!aborted && s.ids[u.y] >= 0 && rA < u.w) {
                const uint8_t *base = s.stages + (size_t)st * p.stage_bytes;
                const uint8_t *rowA = base + (size_t)rA * gu_row_bytes;
                const uint8_t *rowB = base + (size_t)min(rB, u.w - 1) * gu_row_bytes;
                if (p.gu_type == MMRS_Q5K) {
                    vA = row_dot<MMRS_Q5K>(rowA, lig, L, ntasks, ta);
                    vB = row_dot<MMRS_Q5K>(rowB, lig, L, ntasks, ta);
                } else {
                    vA = row_dot<MMRS_Q4K>(rowA, lig, L, ntasks, ta);
                    vB = row_dot<MMRS_Q4K>(rowB, lig, L, ntasks, ta);
                }
            }
#pragma unroll
            for (int m = 16; m > 0; m >>= 1)
                if (m < L) {
                    vA += __shfl_xor_sync(0xffffffffu, vA, m);
                    vB += __shfl_xor_sync(0xffffffffu, vB, m);
                }
            __syncwarp();
            if (lane == 0) mbar_arrive(&s.empty[st]);
            if (lig == 0) {
                float *gv = (u.x == 0 ? s.gval : s.uval) + s.unit_off[k];
                if (rA < u.w) gv[rA] = vA;
                if (rB < u.w) gv[rB] = vB;
            }
        }
        named_sync(1, kConsumerThreads);
        // act = up * silu(gate) (moe_gguf.cu:272-273) for the CTA's whole range
        for (int i = tid; i < gu_p1 - gu_p0; i += kConsumerThreads) {
            const float g = s.gval[i];
            const int slot = s.vslot[(gu_p0 + i) / I];
            s.act_s[i] = (!aborted && s.ids[slot] >= 0) ? s.uval[i] * __fdiv_rn(g, 1.0f + expf(-g)) : 0.f;
        }
        // Q8_1 of act (quantize_silu_mul_q8_1, moe_gguf.cu:255-284) per 32-row block.  Blocks inside
        // this CTA's range are quantised from shared memory; a block shared with neighbour CTAs is
        // published through global scratch and quantised by whichever CTA completes it (one
        // acq_rel arrival per CTA and block).
        named_sync(1, kConsumerThreads);
        if (gu_p1 > gu_p0) {
            const int b_first = gu_p0 >> 5, b_last = (gu_p1 - 1) >> 5;
            for (int b = b_first + warp; b <= b_last; b += kConsumerWarps) {
                const int r = b * 32 + lane;
                const bool inside = r >= gu_p0 && r < gu_p1;
                const int lo = max(b * 32, gu_p0), hi = min(b * 32 + 32, gu_p1);
                bool mine = true;
                if (hi - lo < 32) {
                    if (inside) p.act[r] = s.act_s[r - gu_p0];
                    __syncwarp();
                    uint32_t old = 0;
                    if (lane == 0)
                        asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;"
                                     : "=r"(old)
                                     : "l"(p.blk_count + b), "r"((uint32_t)(hi - lo))
                                     : "memory");
                    old = __shfl_sync(0xffffffffu, old, 0);
                    mine = old + (uint32_t)(hi - lo) == 32u;
                    __syncwarp();
                }
                if (mine && !aborted) {
                    const float v32 = inside ? s.act_s[r - gu_p0] : __ldcg(p.act + r);
                    const float amax = warp_max_butterfly(fabsf(v32));
                    const float dd = __fdiv_rn(amax, 127.0f);
                    const int q = amax == 0.f ? 0 : (int)roundf(__fdiv_rn(v32, dd));
                    int sq = q;
#pragma unroll
                    for (int m = 16; m > 0; m >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, m);
                    p.aq[r] = (int8_t)q;
                    if (lane == 0) {
                        p.ad[b] = __half2float(__float2half_rn(dd));
                        p.aS[b] = sq;
                    }
                }
            }
        }
    }

    // P3: grid barrier, activation copy, down.
    if (tid == 0 && p.trace) p.trace[cta * 16 + 4] = globaltimer_ns();
    const bool sync_ok = grid_sync(p.ctl, (uint32_t)G * (epoch + 2u), deadline, s.flag, 7, kConsumerThreads);
    if (!sync_ok) aborted = true;
    if (tid == 0) {
        if (sync_ok) p.ctl->epoch[cta] = epoch + 2u;  // read again only by this CTA's next launch
        if (p.trace) p.trace[cta * 16 + 5] = globaltimer_ns();
    }
    {
        // One bulk copy of the quantised activation [8][I] (+ scales, sums) per CTA.  Issue and
        // wait depend only on the CTA-uniform barrier result, so the copy has always landed
        // before any consumer thread moves on.
        const uint32_t qb = (uint32_t)(kTopK * I), sb = (uint32_t)(sizeof(float) * kTopK * (I / 32));
        if (tid == 0 && sync_ok) {
            asm volatile("fence.proxy.async;" ::: "memory");  // generic writes -> async-proxy reads
            mbar_arrive_expect_tx(s.abar, qb + 2 * sb);
            bulk_g2s(s.aq_s, p.aq, qb, s.abar);
            bulk_g2s(s.ad_s, p.ad, sb, s.abar);
            bulk_g2s(s.aS_s, p.aS, sb, s.abar);
        }
        if (sync_ok && !mbar_wait_bounded(s.abar, 0u, deadline + 1000000000ull)) {
            atomicExch(&p.ctl->status, (uint32_t)MMRS_ERR_TIMEOUT);
            aborted = true;
        }
        build_task_scales(s.ats, s.ad_s, s.aS_s, kTopK * (I / 64), tid, kConsumerThreads);
        named_sync(1, kConsumerThreads);
        if (tid == 0 && p.trace) p.trace[cta * 16 + 6] = globaltimer_ns();

        // Down units: U_dn rows x all 8 routed experts.  A lane group of L lanes computes one expert
        // (slot) for two rows, with that slot's activation in registers.
        const int L = p.dn_lanes;
        const int q = gw * (32 / L) + lane / L, lig = lane % L;
        const int slot = q % kTopK, rA = (q / kTopK) * kRowsPerLane, rB = rA + 1;
        const int ntasks = (I / QK_K) * 4;
        TaskAct ta[kTPL];
        const int vp = s.vpos[slot];  // position block of this slot's activation
        load_task_acts(ActView{s.aq_s + (size_t)vp * I, s.ats + vp * (I / 64)}, lig, L, ntasks, ta);
        const float wslot = s.w[slot];
        const bool valid = s.ids[slot] >= 0;
        const int j0 = ((grp - n_gu) % kGroups + kGroups) % kGroups;
        for (int k = n_gu + j0; k < n_units; k += kGroups) {
            const int4 u = s.units[k];
            const int st = k % p.stages;
            if (!aborted && !wait_unit(s.full, s.ticket, k, st, p.stages, deadline)) {
                atomicExch(&p.ctl->status, (uint32_t)MMRS_ERR_TIMEOUT);
                aborted = true;
            }
            float vA = 0.f, vB = 0.f;
            if (valid && !aborted && rA < u.w) {
                const uint8_t *base = s.stages + (size_t)st * p.stage_bytes + (size_t)slot * dn_row_bytes * U_dn;
                const uint8_t *rowA = base + (size_t)rA * dn_row_bytes;
                const uint8_t *rowB = base + (size_t)min(rB, u.w - 1) * dn_row_bytes;
                if (p.dn_type == MMRS_Q5K) {
                    vA = row_dot<MMRS_Q5K>(rowA, lig, L, ntasks, ta);
                    vB = row_dot<MMRS_Q5K>(rowB, lig, L, ntasks, ta);
                } else {
                    vA = row_dot<MMRS_Q4K>(rowA, lig, L, ntasks, ta);
                    vB = row_dot<MMRS_Q4K>(rowB, lig, L, ntasks, ta);
                }
            }
#pragma unroll
            for (int m = 16; m > 0; m >>= 1)
                if (m < L) {
                    vA += __shfl_xor_sync(0xffffffffu, vA, m);
                    vB += __shfl_xor_sync(0xffffffffu, vB, m);
                }
            __syncwarp();
            if (lane == 0) mbar_arrive(&s.empty[st]);
            if (lig == 0) {
                const int off = s.unit_off[k];
                if (rA < u.w) s.dn_acc[(off + rA) * kTopK + slot] = valid ? vA * wslot : 0.f;
                if (rB < u.w) s.dn_acc[(off + rB) * kTopK + slot] = valid ? vB * wslot : 0.f;
            }
        }
        // y = fixed 8-way tree over the routed experts (moe_gguf.cu:328-342) + residual
        named_sync(1, kConsumerThreads);
        if (p.world <= 1) {
            for (int r = tid; r < dn_r1 - dn_r0; r += kConsumerThreads) {
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
            for (int r = tid; r < dn_r1 - dn_r0; r += kConsumerThreads) {
                const float *q = s.dn_acc + r * kTopK;
                mine[dn_r0 + r] = ((q[0] + q[4]) + (q[2] + q[6])) + ((q[1] + q[5]) + (q[3] + q[7]));
            }
            named_sync(1, kConsumerThreads);
            if (tid == 0) {
                st_release_sys(reinterpret_cast<uint32_t *>(p.xch + kXchDFlags) + cta, token);
                const uint64_t xdl = globaltimer_ns() + p.timeout_ns;
                for (int rk = 0; rk < p.world; ++rk) {
                    if (rk == p.rank) continue;
                    if (!wait_flag_sys(reinterpret_cast<const uint32_t *>(p.xpeer[rk] + kXchDFlags) + cta, token, xdl)) {
                        atomicExch(&p.ctl->status, (uint32_t)MMRS_ERR_TIMEOUT);
                        atomicExch(reinterpret_cast<uint32_t *>(p.xch + kXchStatus), (uint32_t)MMRS_ERR_TIMEOUT);
                        s.flag[1] = 1;
                        break;
                    }
                }
            }
            named_sync(1, kConsumerThreads);
            const bool xfail = *reinterpret_cast<volatile int *>(&s.flag[1]) != 0;
            for (int r = tid; r < dn_r1 - dn_r0 && !xfail; r += kConsumerThreads) {
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
    }
    if (tid == 0 && p.trace) p.trace[cta * 16 + 7] = globaltimer_ns();
}

// ------------------------------------------------------------------------------------------
// Host side
// ------------------------------------------------------------------------------------------
size_t decode_smem_bytes(const DecodeParams &p) {
    auto a16 = [](size_t v) { return (v + 15) / 16 * 16; };
    size_t b = a16((size_t)p.stages * p.stage_bytes) + 2 * a16(sizeof(uint64_t) * p.stages) + a16(8);
    b += a16(p.H) + 2 * a16(4 * (p.H / 32)) + a16(16 * (p.H / 64));
    b += a16((size_t)kTopK * p.I) + 2 * a16(4 * kTopK * (p.I / 32)) + a16(16 * kTopK * (p.I / 64));
    b += a16(4 * (p.E > 16 ? p.E : 16)) + a16(4 * p.E) + 4 * a16(4 * kTopK);  // part, sig, ids, vslot, vpos, w
    b += a16(4 * p.res_slots * kTopK) + 3 * a16(4 * p.act_slots) + a16(4 * p.res_slots) + 32;
    b += a16(16 * kMaxUnits) + a16(4 * kMaxUnits) + 16 + a16(4 * p.stages);
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
    if (p.H / 128 > 2 * kConsumerWarps || p.H / 8 / 4 > 128) return MMRS_ERR_UNSUPPORTED;  // H <= 4096
    const int gu_tasks = (p.H / QK_K) * 4, dn_tasks = (p.I / QK_K) * 4;
    p.gu_lanes = pow2_at_least((gu_tasks + kTPL - 1) / kTPL);
    p.dn_lanes = pow2_at_least((dn_tasks + kTPL - 1) / kTPL);
    if (p.gu_lanes > 16 || p.dn_lanes > 32) return MMRS_ERR_UNSUPPORTED;  // H <= 3072, I <= 6144
    // units: kGroupWarps warps x (32/L) lane groups x kRowsPerLane rows
    p.gu_unit_rows = kGroupWarps * (32 / p.gu_lanes) * kRowsPerLane;
    p.dn_unit_rows = kGroupWarps * (32 / p.dn_lanes) * kRowsPerLane / kTopK;
    if (p.dn_unit_rows < kRowsPerLane) return MMRS_ERR_UNSUPPORTED;
    p.act_slots = (kTopK * p.I + num_sms - 1) / num_sms + 1;
    p.res_slots = (p.H + num_sms - 1) / num_sms + 1;
    if (p.res_slots > kConsumerThreads || p.E > 2 * num_sms) return MMRS_ERR_UNSUPPORTED;
    const int max_gu_units = 2 * ((p.act_slots + p.gu_unit_rows - 1) / p.gu_unit_rows + kTopK);
    const int max_dn_units = (p.res_slots + p.dn_unit_rows - 1) / p.dn_unit_rows;
    if (max_gu_units + max_dn_units > kMaxUnits) return MMRS_ERR_UNSUPPORTED;
    const size_t gu_stage = kq_row_bytes(p.gu_type, p.H) * p.gu_unit_rows;
    const size_t dn_stage = kq_row_bytes(p.dn_type, p.I) * p.dn_unit_rows * kTopK;
    p.stage_bytes = (int)(((gu_stage > dn_stage ? gu_stage : dn_stage) + 127) / 128 * 128);
    p.stages = 0;
    DecodeParams q = p;
    for (int st = 16; st >= 2; --st) {
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
    cudaError_t err = cudaSuccess;
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
    err = cudaLaunchKernelEx(&cfg, moe_decode_fused_kernel, p);
    return err == cudaSuccess ? MMRS_OK : MMRS_ERR_LAUNCH;
}

}  // namespace mmrs
