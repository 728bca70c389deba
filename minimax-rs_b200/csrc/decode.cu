// Fused single-token MoE block for B200 (sm_100a).
//
// Replaces, in one persistent launch, the reference's decode chain
//   router Linear (fused_moe.rs:267) -> minimax_moe_decode_topk (moe_gguf.cu:34-100)
//   -> quantize_q8_1 -> moe_gate_up_decode_kernel -> quantize_silu_mul_q8_1
//   -> moe_down_decode_kernel (moe_gguf.cu:200-343, 426-567) -> + residual (model.rs:218)
//
// Design (one CTA per SM, 8 consumer warps + 1 producer warp):
//   P0  router GEMV: expert e is computed by warp (e / grid) of CTA (e % grid) in the library's
//       canonical order (32 lane partials of float4 groups, fmaf, xor butterfly).  Meanwhile every
//       CTA quantises x to Q8_1 in shared memory.  Grid barrier #1.
//   P1  every CTA redundantly selects the top-8 from the 256 logits (sigmoid + bias, stable
//       descending rank) and renormalises the weights with the reference's fixed tree.
//   P2  gate/up: units of R=4 rows x {gate, up} of one routed expert; each CTA owns a contiguous
//       unit range.  The producer streams units into a ring of shared-memory stages with 1-D bulk
//       TMA copies (cp.async.bulk + mbarrier complete_tx); 8 warps = 4 rows x {gate, up} consume,
//       and the gate warp of each pair writes act = up * silu(gate) (f32) to global scratch.
//   P3  down: units of Rd rows x 8 routed experts.  The producer keeps streaming (down weights do
//       not depend on act), so down tiles are already resident when grid barrier #2 releases.  Each
//       CTA quantises act to Q8_1 in shared memory, warp w handles slot w, and the 8 slot values of
//       each row are summed with the reference's tree ((v0+v4)+(v2+v6))+((v1+v5)+(v3+v7)).
// Every wait (mbarrier, grid barrier) is bounded by a globaltimer deadline; on expiry the kernel
// records MMRS_ERR_TIMEOUT in the workspace status word, drains its own copies and returns.
#include "common.cuh"
#include "decode.cuh"

namespace mmrs {

constexpr int kConsumerWarps = 8;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kTopK = 8;
constexpr int kMaxTPL = 4;  // tasks per lane (a task = 16 bytes of quants of one super-block)

// Shared-memory activation in Q8_1 form: int8 q[K], float d[K/32], int s16[K/16] (sums of halves).
struct ActView {
    int8_t *q;
    float *d;
    int *s16;
};

// Per-lane register copy of the activation slices its tasks touch.
struct LaneAct {
    int lo[kMaxTPL][4], hi[kMaxTPL][4];
    float dlo[kMaxTPL], dhi[kMaxTPL];
    int slo[kMaxTPL], shi[kMaxTPL];
};

__device__ __forceinline__ void load_lane_act(const ActView &a, int lane_in_group, int group_lanes,
                                              int ntasks, LaneAct &la) {
#pragma unroll
    for (int i = 0; i < kMaxTPL; ++i) {
        const int tau = lane_in_group + group_lanes * i;
        if (tau < ntasks) {
            const int b = tau >> 3, t = tau & 7, j = t >> 1, h = t & 1;
            const int elo = 256 * b + 64 * j + 16 * h, ehi = elo + 32;
            const int4 vlo = *reinterpret_cast<const int4 *>(a.q + elo);
            const int4 vhi = *reinterpret_cast<const int4 *>(a.q + ehi);
            la.lo[i][0] = vlo.x; la.lo[i][1] = vlo.y; la.lo[i][2] = vlo.z; la.lo[i][3] = vlo.w;
            la.hi[i][0] = vhi.x; la.hi[i][1] = vhi.y; la.hi[i][2] = vhi.z; la.hi[i][3] = vhi.w;
            la.dlo[i] = a.d[elo >> 5];
            la.dhi[i] = a.d[ehi >> 5];
            la.slo[i] = a.s16[elo >> 4];
            la.shi[i] = a.s16[ehi >> 4];
        } else {
#pragma unroll
            for (int c = 0; c < 4; ++c) la.lo[i][c] = la.hi[i][c] = 0;
            la.dlo[i] = la.dhi[i] = 0.f;
            la.slo[i] = la.shi[i] = 0;
        }
    }
}

// Partial dot of one row (in shared memory) against the lane's activation slices, MMVQ formula
// of vec_dot_q4_K_q8_1 / vec_dot_q5_K_q8_1 (gguf.cuh:727-750, 783-813): per super-block
// dall * sum d8*(dot*sc) - dmin * sum d8*(sumq*m).
template <int TYPE>
__device__ __forceinline__ float row_partial(const uint8_t *row, int lane_in_group, int group_lanes,
                                             int ntasks, const LaneAct &la) {
    constexpr int BB = TYPE == MMRS_Q5K ? Q5K_BYTES : Q4K_BYTES;
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxTPL; ++i) {
        const int tau = lane_in_group + group_lanes * i;
        if (tau < ntasks) {
            const int b = tau >> 3, t = tau & 7, j = t >> 1, h = t & 1;
            const uint8_t *blk = row + b * BB;
            const uint4 hdr = *reinterpret_cast<const uint4 *>(blk);
            uint4 qv;
            int vlo[4], vhi[4];
            if (TYPE == MMRS_Q5K) {
                qv = *reinterpret_cast<const uint4 *>(blk + 48 + 32 * j + 16 * h);
                const uint4 qh = *reinterpret_cast<const uint4 *>(blk + 16 + 16 * h);
                const uint32_t q[4] = {qv.x, qv.y, qv.z, qv.w};
                const uint32_t hb[4] = {qh.x, qh.y, qh.z, qh.w};
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    vlo[c] = (int)((q[c] & 0x0F0F0F0Fu) | (((hb[c] >> (2 * j)) & 0x01010101u) << 4));
                    vhi[c] = (int)(((q[c] >> 4) & 0x0F0F0F0Fu) | (((hb[c] >> (2 * j + 1)) & 0x01010101u) << 4));
                }
            } else {
                qv = *reinterpret_cast<const uint4 *>(blk + 16 + 32 * j + 16 * h);
                const uint32_t q[4] = {qv.x, qv.y, qv.z, qv.w};
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    vlo[c] = (int)(q[c] & 0x0F0F0F0Fu);
                    vhi[c] = (int)((q[c] >> 4) & 0x0F0F0F0Fu);
                }
            }
            int dlo = 0, dhi = 0;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                dlo = __dp4a(vlo[c], la.lo[i][c], dlo);
                dhi = __dp4a(vhi[c], la.hi[i][c], dhi);
            }
            int sc0, m0, sc1, m1;
            kq_scale_min_pair(hdr.y, hdr.z, hdr.w, j, sc0, m0, sc1, m1);
            const float sd = la.dlo[i] * (float)(dlo * sc0) + la.dhi[i] * (float)(dhi * sc1);
            const float sm = la.dlo[i] * (float)(la.slo[i] * m0) + la.dhi[i] * (float)(la.shi[i] * m1);
            const float dall = half_bits_to_float(hdr.x), dmin = half_bits_to_float(hdr.x >> 16);
            acc += dall * sd - dmin * sm;
        }
    }
    return acc;
}

// Quantise 32 values held one per lane into Q8_1 (quantize_q8_1, gguf.cuh:1234-1261;
// quantize_silu_mul_q8_1, moe_gguf.cu:255-284): d = amax/127, q = roundf(v/d).
// Writes q (lane), d and the two 16-lane sums.
__device__ __forceinline__ void warp_quant_q81(float v, int8_t *q, float *d, int *s16, int lane) {
    const float amax = warp_max_butterfly(fabsf(v));
    const float dd = __fdiv_rn(amax, 127.0f);
    const int qi = amax == 0.f ? 0 : (int)roundf(__fdiv_rn(v, dd));
    q[lane] = (int8_t)qi;
    int s = qi;
#pragma unroll
    for (int m = 8; m > 0; m >>= 1) s += __shfl_xor_sync(0xffffffffu, s, m);
    if (lane == 0) {
        *d = __half2float(__float2half_rn(dd));
        s16[0] = s;
    }
    if (lane == 16) s16[1] = s;
}

struct DecodeSmem {
    // carved from dynamic shared memory by the kernel
    uint8_t *stages;
    uint64_t *full, *empty;
    float *x;  // [H]
    ActView xq, aq;  // aq: [8][I] q, [8][I/32] d, [8][I/16] s16
    float *sel, *sig;  // [E]
    int *ids;          // [8]
    float *w;          // [8]
    float *gu_vals;    // [2][4][2]
    float *dn_vals;    // [2][8 rows max][8]
    int *flag;
};

__global__ void __launch_bounds__(kThreads, 1) moe_decode_fused_kernel(const __grid_constant__ DecodeParams p) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, cta = blockIdx.x;
    const int H = p.H, I = p.I, E = p.E;
    const uint64_t deadline = globaltimer_ns() + p.timeout_ns;

    // ---- carve shared memory ------------------------------------------------------------
    DecodeSmem s;
    {
        uint8_t *ptr = smem_raw;
        s.stages = ptr;
        ptr += (size_t)p.stages * p.stage_bytes;
        s.full = reinterpret_cast<uint64_t *>(ptr);
        ptr += sizeof(uint64_t) * p.stages;
        s.empty = reinterpret_cast<uint64_t *>(ptr);
        ptr += sizeof(uint64_t) * p.stages;
        s.x = reinterpret_cast<float *>(ptr);
        ptr += sizeof(float) * H;
        s.xq.q = reinterpret_cast<int8_t *>(ptr);
        ptr += H;
        s.xq.d = reinterpret_cast<float *>(ptr);
        ptr += sizeof(float) * (H / 32);
        s.xq.s16 = reinterpret_cast<int *>(ptr);
        ptr += sizeof(int) * (H / 16);
        s.aq.q = reinterpret_cast<int8_t *>(ptr);
        ptr += (size_t)kTopK * I;
        s.aq.d = reinterpret_cast<float *>(ptr);
        ptr += sizeof(float) * kTopK * (I / 32);
        s.aq.s16 = reinterpret_cast<int *>(ptr);
        ptr += sizeof(int) * kTopK * (I / 16);
        s.sel = reinterpret_cast<float *>(ptr);
        ptr += sizeof(float) * E;
        s.sig = reinterpret_cast<float *>(ptr);
        ptr += sizeof(float) * E;
        s.ids = reinterpret_cast<int *>(ptr);
        ptr += sizeof(int) * kTopK;
        s.w = reinterpret_cast<float *>(ptr);
        ptr += sizeof(float) * kTopK;
        s.gu_vals = reinterpret_cast<float *>(ptr);
        ptr += sizeof(float) * 16;
        s.dn_vals = reinterpret_cast<float *>(ptr);
        ptr += sizeof(float) * 2 * 8 * kTopK;
        s.flag = reinterpret_cast<int *>(ptr);
    }
    if (tid == 0) {
        for (int i = 0; i < p.stages; ++i) {
            mbar_init(&s.full[i], 1);
            mbar_init(&s.empty[i], kConsumerWarps);
        }
        fence_mbar_init();
        s.flag[0] = 1;  // ok
    }
    __syncthreads();

    const int gu_units_begin = (int)((int64_t)cta * p.n_gu_units / G);
    const int gu_units_end = (int)((int64_t)(cta + 1) * p.n_gu_units / G);
    const int dn_units_begin = (int)((int64_t)cta * p.n_dn_units / G);
    const int dn_units_end = (int)((int64_t)(cta + 1) * p.n_dn_units / G);
    const int n_gu = gu_units_end - gu_units_begin, n_dn = dn_units_end - dn_units_begin;
    const int gu_units_per_slot = I / p.gu_rows;
    const size_t gu_row_bytes = kq_row_bytes(p.gu_type, H);
    const size_t dn_row_bytes = kq_row_bytes(p.dn_type, I);
    const size_t gu_expert_bytes = gu_row_bytes * I;
    const size_t dn_expert_bytes = dn_row_bytes * H;

    // ---- P0: x -> smem, router GEMV, Q8_1 of x --------------------------------------------
    if (warp < kConsumerWarps) {
        for (int i = tid; i < H / 4; i += kConsumerWarps * 32)
            reinterpret_cast<float4 *>(s.x)[i] = __ldg(reinterpret_cast<const float4 *>(p.x) + i);
        named_sync(1, kConsumerWarps * 32);
        if (p.internal_routing) {
            for (int e = cta + G * warp; e < E; e += G * kConsumerWarps) {
                const float4 *wr = reinterpret_cast<const float4 *>(p.router + (size_t)e * H);
                const float4 *xv = reinterpret_cast<const float4 *>(s.x);
                float acc = 0.f;
                for (int i = lane; i < H / 4; i += 32) {
                    const float4 w4 = __ldg(wr + i);
                    const float4 x4 = xv[i];
                    acc = fmaf(w4.x, x4.x, acc);
                    acc = fmaf(w4.y, x4.y, acc);
                    acc = fmaf(w4.z, x4.z, acc);
                    acc = fmaf(w4.w, x4.w, acc);
                }
                acc = warp_sum_butterfly(acc);
                if (lane == 0) p.logits[e] = acc;
            }
        }
        for (int b = warp; b < H / 32; b += kConsumerWarps)
            warp_quant_q81(s.x[b * 32 + lane], s.xq.q + b * 32, s.xq.d + b, s.xq.s16 + 2 * b, lane);
    }

    // ---- P1: routing (all CTAs redundantly) -----------------------------------------------
    bool ok = true;
    if (p.internal_routing) {
        ok = grid_barrier(p.bar, G, deadline, s.flag, 2, kThreads);
        if (ok) {
            for (int e = tid; e < E; e += kThreads) {
                const float l = __ldcg(p.logits + e);
                const float sg = __fdiv_rn(1.0f, 1.0f + expf(-l));
                s.sig[e] = sg;
                s.sel[e] = sg + p.bias[e];
            }
            __syncthreads();
            for (int e = tid; e < E; e += kThreads) {
                const float me = s.sel[e];
                int rank = 0;
                for (int j = 0; j < E; ++j) {
                    const float o = s.sel[j];
                    rank += (o > me) || (o == me && j < e);
                }
                if (rank < kTopK) s.ids[rank] = e;
            }
            __syncthreads();
            if (tid == 0) {
                float v[kTopK];
                for (int k = 0; k < kTopK; ++k) v[k] = s.sig[s.ids[k]];
                const float a0 = v[0] + v[4], a1 = v[1] + v[5], a2 = v[2] + v[6], a3 = v[3] + v[7];
                const float denom = (a0 + a2) + (a1 + a3);
                for (int k = 0; k < kTopK; ++k) s.w[k] = __fdiv_rn(v[k], denom);
            }
            __syncthreads();
            if (cta == 0 && tid < kTopK) {
                if (p.topk_ids_out) p.topk_ids_out[tid] = (uint32_t)s.ids[tid];
                if (p.topk_w_out) p.topk_w_out[tid] = s.w[tid];
            }
        }
    } else {
        if (tid < kTopK) {
            s.ids[tid] = -1;
            s.w[tid] = 0.f;
        }
        __syncthreads();
        if (tid < kTopK) {
            // pairs (route, expert) in expert order; routes outside [0, 8) and invalid experts
            // contribute nothing, as in moe_down_decode_kernel (moe_gguf.cu:311)
            const int slot = p.ext_route[tid];
            const int e = p.ext_expert[tid];
            if (slot >= 0 && slot < kTopK) {
                s.ids[slot] = (e >= 0 && e < E) ? e : -1;
                s.w[slot] = p.ext_w[slot];
            }
        }
        __syncthreads();
    }

    if (!ok) {
        // nothing was issued yet: just leave
        return;
    }

    if (warp == kConsumerWarps) {
        // ---------------------------- producer --------------------------------------------
        if (lane == 0) {
            int it = 0;
            bool pok = true;
            const int total = n_gu + n_dn;
            for (; it < total && pok; ++it) {
                const int st = it % p.stages;
                const uint32_t ph = (uint32_t)(it / p.stages) & 1u;
                if (!mbar_wait_bounded(&s.empty[st], ph ^ 1u, deadline)) {
                    pok = false;
                    atomicExch(&p.bar->status, (uint32_t)MMRS_ERR_TIMEOUT);
                    break;
                }
                uint8_t *dst = s.stages + (size_t)st * p.stage_bytes;
                if (it < n_gu) {
                    const int u = gu_units_begin + it;
                    const int slot = u / gu_units_per_slot;
                    const int row0 = (u % gu_units_per_slot) * p.gu_rows;
                    const int e = s.ids[slot];
                    const uint32_t bytes = (uint32_t)(gu_row_bytes * p.gu_rows);
                    if (e >= 0) {
                        mbar_arrive_expect_tx(&s.full[st], 2 * bytes);
                        const size_t off = (size_t)e * gu_expert_bytes + (size_t)row0 * gu_row_bytes;
                        bulk_g2s(dst, p.gate + off, bytes, &s.full[st]);
                        bulk_g2s(dst + bytes, p.up + off, bytes, &s.full[st]);
                    } else {
                        mbar_arrive(&s.full[st]);
                    }
                } else {
                    const int u = dn_units_begin + (it - n_gu);
                    const int row0 = u * p.dn_rows;
                    const uint32_t bytes = (uint32_t)(dn_row_bytes * p.dn_rows);
                    uint32_t tx = 0;
                    for (int k = 0; k < kTopK; ++k) tx += s.ids[k] >= 0 ? bytes : 0;
                    mbar_arrive_expect_tx(&s.full[st], tx);
                    for (int k = 0; k < kTopK; ++k) {
                        const int e = s.ids[k];
                        if (e < 0) continue;
                        bulk_g2s(dst + (size_t)k * bytes,
                                 p.down + (size_t)e * dn_expert_bytes + (size_t)row0 * dn_row_bytes, bytes,
                                 &s.full[st]);
                    }
                }
            }
            // Drain: make sure no copy is still landing in shared memory when the CTA retires.
            const int first = it > p.stages ? it - p.stages : 0;
            for (int j = first; j < it; ++j)
                mbar_wait_bounded(&s.full[j % p.stages], (uint32_t)(j / p.stages) & 1u, deadline + 1000000000ull);
        }
        return;
    }

    // ------------------------------- consumers ----------------------------------------------
    // P2: gate/up.  warp w -> row (w >> 1) of the unit, matrix (w & 1): 0 = gate, 1 = up.
    bool aborted = false;
    const int gu_tasks = (H / QK_K) * 8;
    {
        LaneAct la;
        load_lane_act(s.xq, lane, 32, gu_tasks, la);
        const int r = warp >> 1, mat = warp & 1;
        for (int it = 0; it < n_gu; ++it) {
            const int st = it % p.stages;
            // On a timeout keep iterating without waiting so every named barrier still matches.
            if (!aborted && !mbar_wait_bounded(&s.full[st], (uint32_t)(it / p.stages) & 1u, deadline)) {
                atomicExch(&p.bar->status, (uint32_t)MMRS_ERR_TIMEOUT);
                aborted = true;
            }
            const int u = gu_units_begin + it;
            const int slot = u / gu_units_per_slot;
            const int row = (u % gu_units_per_slot) * p.gu_rows + r;
            const uint8_t *src = s.stages + (size_t)st * p.stage_bytes + (size_t)mat * gu_row_bytes * p.gu_rows +
                                 (size_t)r * gu_row_bytes;
            float v = 0.f;
            if (!aborted && s.ids[slot] >= 0)
                v = p.gu_type == MMRS_Q5K ? row_partial<MMRS_Q5K>(src, lane, 32, gu_tasks, la)
                                          : row_partial<MMRS_Q4K>(src, lane, 32, gu_tasks, la);
            v = warp_sum_butterfly(v);
            __syncwarp();
            if (lane == 0) mbar_arrive(&s.empty[st]);
            float *gv = s.gu_vals + (it & 1) * 8;
            if (lane == 0) gv[r * 2 + mat] = v;
            named_sync(3 + r, 64);
            if (mat == 0 && lane == 0) {
                const float g = gv[r * 2 + 0], up = gv[r * 2 + 1];
                p.act[(size_t)slot * I + row] = up * __fdiv_rn(g, 1.0f + expf(-g));
            }
        }
    }

    // P3: grid barrier, quantise act, down.
    if (!grid_barrier(p.bar, G, deadline, s.flag, 7, kConsumerWarps * 32)) aborted = true;
    for (int b = warp; b < kTopK * (I / 32); b += kConsumerWarps) {
        const int slot = b / (I / 32), bb = b % (I / 32);
        const float v = __ldcg(p.act + (size_t)slot * I + bb * 32 + lane);
        warp_quant_q81(v, s.aq.q + (size_t)slot * I + bb * 32, s.aq.d + slot * (I / 32) + bb,
                       s.aq.s16 + slot * (I / 16) + 2 * bb, lane);
    }
    named_sync(1, kConsumerWarps * 32);
    {
        const int dn_tasks = (I / QK_K) * 8;
        const int group_lanes = 32 / p.dn_rows;
        const int grp = lane / group_lanes, lig = lane % group_lanes;
        const int slot = warp;
        LaneAct la;
        const ActView aslot = {s.aq.q + (size_t)slot * I, s.aq.d + slot * (I / 32), s.aq.s16 + slot * (I / 16)};
        load_lane_act(aslot, lig, group_lanes, dn_tasks, la);
        const float wslot = s.w[slot];
        const bool valid = s.ids[slot] >= 0;
        for (int j = 0; j < n_dn; ++j) {
            const int it = n_gu + j;
            const int st = it % p.stages;
            if (!aborted && !mbar_wait_bounded(&s.full[st], (uint32_t)(it / p.stages) & 1u, deadline)) {
                atomicExch(&p.bar->status, (uint32_t)MMRS_ERR_TIMEOUT);
                aborted = true;
            }
            const uint8_t *src = s.stages + (size_t)st * p.stage_bytes + (size_t)slot * dn_row_bytes * p.dn_rows +
                                 (size_t)grp * dn_row_bytes;
            float v = 0.f;
            if (valid && !aborted)
                v = p.dn_type == MMRS_Q5K ? row_partial<MMRS_Q5K>(src, lig, group_lanes, dn_tasks, la)
                                          : row_partial<MMRS_Q4K>(src, lig, group_lanes, dn_tasks, la);
#pragma unroll
            for (int m = 16; m > 0; m >>= 1)
                if (m < group_lanes) v += __shfl_xor_sync(0xffffffffu, v, m);
            __syncwarp();
            if (lane == 0) mbar_arrive(&s.empty[st]);
            float *dv = s.dn_vals + (j & 1) * 8 * kTopK;
            if (lig == 0) dv[grp * kTopK + slot] = valid ? v * wslot : 0.f;
            named_sync(1, kConsumerWarps * 32);
            if (warp == 0 && lane < p.dn_rows) {
                const float *q = dv + lane * kTopK;
                float y = ((q[0] + q[4]) + (q[2] + q[6])) + ((q[1] + q[5]) + (q[3] + q[7]));
                const int row = (dn_units_begin + j) * p.dn_rows + lane;
                if (p.residual) y = y + p.residual[row];
                p.y[row] = y;
            }
        }
    }
}

// ------------------------------------------------------------------------------------------
// Host side
// ------------------------------------------------------------------------------------------
size_t decode_smem_bytes(const DecodeParams &p) {
    size_t b = (size_t)p.stages * p.stage_bytes + 2 * sizeof(uint64_t) * p.stages;
    b += sizeof(float) * p.H + p.H + sizeof(float) * (p.H / 32) + sizeof(int) * (p.H / 16);
    b += (size_t)kTopK * (p.I + sizeof(float) * (p.I / 32) + sizeof(int) * (p.I / 16));
    b += 2 * sizeof(float) * p.E + 2 * sizeof(int) * kTopK + sizeof(float) * (16 + 2 * 8 * kTopK) + 16;
    return b;
}

int decode_configure(DecodeParams &p, int num_sms, int max_smem) {
    if (p.H % QK_K || p.I % QK_K || p.H > 4096 || p.E > 1024 || p.E < kTopK) return MMRS_ERR_UNSUPPORTED;
    if ((p.gu_type != MMRS_Q4K && p.gu_type != MMRS_Q5K) || (p.dn_type != MMRS_Q4K && p.dn_type != MMRS_Q5K))
        return MMRS_ERR_UNSUPPORTED;
    const int dn_blocks = p.I / QK_K;
    if (dn_blocks > 16) return MMRS_ERR_UNSUPPORTED;
    p.gu_rows = 4;
    // rows per down unit so that every lane gets <= kMaxTPL tasks of 16 quant bytes
    int dn_rows = 1;
    for (int r = 8; r >= 1; r /= 2) {
        const int lanes = 32 / r;
        if ((dn_blocks * 8 + lanes - 1) / lanes <= kMaxTPL && p.H % r == 0) {
            dn_rows = r;
            break;
        }
    }
    p.dn_rows = dn_rows;
    if ((dn_blocks * 8 + (32 / dn_rows) - 1) / (32 / dn_rows) > kMaxTPL) return MMRS_ERR_UNSUPPORTED;
    if ((p.H / QK_K) * 8 > 32 * kMaxTPL) return MMRS_ERR_UNSUPPORTED;
    p.n_gu_units = kTopK * (p.I / p.gu_rows);
    p.n_dn_units = p.H / p.dn_rows;
    const size_t gu_stage = 2 * kq_row_bytes(p.gu_type, p.H) * p.gu_rows;
    const size_t dn_stage = kTopK * kq_row_bytes(p.dn_type, p.I) * p.dn_rows;
    p.stage_bytes = (int)(((gu_stage > dn_stage ? gu_stage : dn_stage) + 127) / 128 * 128);
    p.stages = 1;
    DecodeParams q = p;
    for (int st = 16; st >= 2; --st) {
        q.stages = st;
        if (decode_smem_bytes(q) <= (size_t)max_smem) {
            p.stages = st;
            break;
        }
    }
    if (decode_smem_bytes(p) > (size_t)max_smem) return MMRS_ERR_UNSUPPORTED;
    p.grid = num_sms;
    return MMRS_OK;
}

int decode_launch(const DecodeParams &p, cudaStream_t stream) {
    const size_t smem = decode_smem_bytes(p);
    // Raise the dynamic shared-memory limit once per device (the attribute is per context).
    static int configured[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    cudaError_t err = cudaSuccess;
    if (dev < 0 || dev >= 64 || configured[dev] < (int)smem) {
        int optin = 0;
        cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        err = cudaFuncSetAttribute(moe_decode_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, optin);
        if (err != cudaSuccess) return MMRS_ERR_LAUNCH;
        if (dev >= 0 && dev < 64) configured[dev] = optin;
    }
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
