// Single-token attention half of a MiniMax-M2.7 layer on B200 (sm_100a).
//
// Reference path (minimax-rs, src/model.rs:79-162, T = 1): q8_0_decode_rmsnorm_f16
// (candle-nn fused_qkv.rs:162-280 -> mmvq_gguf.cu:814-885), partial_rope_f16
// (mmvq_gguf.cu:1038-1066), KV-cache append, gqa_decode_f16_128 (fused_attention.rs:21-42 ->
// decode_attention.cu:311-918) and the Q8_0 output projection (QMatMul: quantize_q8_1 +
// mmvq, mmvq_gguf.cu:1137-1200).
//
// All of it is memory-bound (Q8_0 weights 46.8 MB and the f16 KV cache per token).  The fused
// forward is three launches chained by programmatic dependent launch:
//   * Q8_0 matvec (dp4a): each CTA quantises the activation into shared memory (8 threads per
//     32-block) and owns a contiguous range of rows, which it asks L2 to fetch before waiting for
//     the previous kernel; a warp takes a row, its lanes stride over the 34-byte blocks read as
//     aligned 32-bit words and realigned with funnel shifts (k % 64 == 0 keeps the last word of
//     every block inside its row);
//   * GQA decode on the tensor cores: CTA = (key split, KV head), K / V chunks streamed by TMA into
//     128-byte-swizzled shared tiles, Q K^T and P V as mma.m16n8k16 with the 6 query heads as M;
//     its prologue does the Q / K RMSNorm, RoPE and the KV append, the last CTA of a KV head merges
//     the splits and writes the Q8_1 blocks the output projection reads;
//   * the output projection (the matvec on ready Q8_1 blocks, + residual).
// The reference-named launchers run the same kernels one operation at a time.
#include <cuda_fp16.h>

#include <algorithm>
#include <cfloat>
#include <mutex>
#include <type_traits>

#include "../../include/minimax_attn.h"
#include "common.cuh"
#include "tma.cuh"
#include "workspace.cuh"

namespace mmrs {

constexpr int kAttnHeadDim = 128;
constexpr int kAttnGroup = 6;            // query heads per KV head
constexpr int kAttnPartial = kAttnHeadDim + 2;  // (max, sum, 128 unnormalised values)
constexpr int kAttnMaxSplits = 128;
constexpr int kMvThreads = 256;          // matvec CTA: 8 warps, one row per warp at a time
constexpr int kMvMaxK = 8192;

// ------------------------------------------------------------------------------------------
// Q8_1 of one 32-element block (quantize_q8_1, mmvq_gguf.cu:1137-1169): lane = element;
// d = amax / 127, q = roundf(x / d); the block's half d (for the dot) and half sum.
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ int8_t q81_lane(float x, float &d_out, float &sum_out) {
    float amax = fabsf(x), sum = x;
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) {
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, m));
        sum += __shfl_xor_sync(0xffffffffu, sum, m);
    }
    const float d = __fdiv_rn(amax, 127.0f);
    d_out = d;
    sum_out = sum;
    return amax == 0.0f ? (int8_t)0 : (int8_t)roundf(__fdiv_rn(x, d));
}

// Activation in shared memory: int8 quants [k] and the per-block half d as float [k / 32].
struct MvAct {
    int8_t *q;
    float *d;
};

// Quantise x (f32 or f16, zero past k) into shared memory, 8 threads per 32-block with 4 values
// each; optionally also store the Q8_1 blocks in the reference's 36-byte layout (vy, kpad / 32
// blocks).  amax and d are those of quantize_q8_1; the block sum pairs elements at distances 16,
// 8, 4 (threads xor 4, 2, 1) then 2 and 1 (inside the thread), the order of lane 0 of the
// reference's 32-lane butterfly, so the stored half sum is bit-identical.
template <typename T>
__device__ void mv_quantize(const T *__restrict__ x, int k, int kpad, MvAct a, uint8_t *vy, int tid, int nthreads) {
    const int nb = kpad / 32;
    for (int base = 0; base < nb * 8; base += nthreads) {  // uniform trip count: shuffles stay converged
        const int t = base + tid, b = t >> 3, j = t & 7, i0 = 32 * b + 4 * j;
        float v[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) v[c] = (t < nb * 8 && i0 + c < k) ? (float)x[i0 + c] : 0.0f;
        float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
        const float d = __fdiv_rn(amax, 127.0f);
        uint32_t packed = 0;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int q = amax == 0.0f ? 0 : (int)roundf(__fdiv_rn(v[c], d));
            packed |= (uint32_t)(q & 0xFF) << (8 * c);
        }
        float sm[4] = {v[0], v[1], v[2], v[3]};
        if (vy) {
#pragma unroll
            for (int m = 4; m > 0; m >>= 1)
#pragma unroll
                for (int c = 0; c < 4; ++c) sm[c] += __shfl_xor_sync(0xffffffffu, sm[c], m);
            sm[0] += sm[2];
            sm[1] += sm[3];
            sm[0] += sm[1];
        }
        if (t < nb * 8) {
            *reinterpret_cast<uint32_t *>(a.q + i0) = packed;
            if (j == 0) a.d[b] = __half2float(__float2half_rn(d));
            if (vy) {
                uint8_t *blk = vy + (size_t)b * 36;
                *reinterpret_cast<uint32_t *>(blk + 4 + 4 * j) = packed;
                if (j == 0)
                    *reinterpret_cast<uint32_t *>(blk) =
                        (uint32_t)__half_as_ushort(__float2half_rn(d)) |
                        ((uint32_t)__half_as_ushort(__float2half_rn(sm[0])) << 16);
            }
        }
    }
}

// Dot of Q8_0 row `row` (nb blocks of 34 bytes, nb even) with the shared-memory activation; lane
// l takes blocks l, l + 32, l + 64, ... (three blocks' words in flight before any arithmetic); the
// result is returned on every lane.
template <bool kShared = false>
__device__ __forceinline__ float mv_row_dot(const uint8_t *__restrict__ row, int nb, MvAct a, int lane) {
    float acc = 0.0f;
    for (int b0 = lane; b0 < nb; b0 += 96) {
        // each block's 34 bytes from 9 aligned words: even b starts on a word, odd b two bytes in
        uint32_t W[3][9];
#pragma unroll
        for (int u = 0; u < 3; ++u) {
            const int b = b0 + 32 * u;
            const uint32_t *w = reinterpret_cast<const uint32_t *>(row + ((34 * b) & ~3));
#pragma unroll
            for (int i = 0; i < 9; ++i) W[u][i] = b < nb ? (kShared ? w[i] : __ldg(w + i)) : 0u;
        }
#pragma unroll
        for (int u = 0; u < 3; ++u) {
            const int b = b0 + 32 * u;
            if (b >= nb) break;
            const bool odd = b & 1;
            const uint32_t sh = odd ? 32u : 16u;
            const float dw =
                __half2float(__ushort_as_half((unsigned short)((odd ? W[u][0] >> 16 : W[u][0]) & 0xFFFFu)));
            const int4 *xq = reinterpret_cast<const int4 *>(a.q + 32 * b);
            const int4 x0 = xq[0], x1 = xq[1];
            const int xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
            int s0 = 0, s1 = 0;
#pragma unroll
            for (int i = 0; i < 8; i += 2) {
                s0 = __dp4a((int)__funnelshift_rc(W[u][i], W[u][i + 1], sh), xv[i], s0);
                s1 = __dp4a((int)__funnelshift_rc(W[u][i + 1], W[u][i + 2], sh), xv[i + 1], s1);
            }
            // vec_dot_q8_0_q8_1_impl (mmvq_gguf.cu:282-290): sumi * d_w * d_x
            acc += __fmul_rn(__fmul_rn((float)(s0 + s1), dw), a.d[b]);
        }
    }
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, m);
    return acc;
}

// One or more Q8_0 matrices sharing one activation: rows [0, n0) of w0, then n1 rows of w1, then
// n2 rows of w2, into dst [n0 + n1 + n2] (+ residual when given).  The activation is x (f32 or
// f16, quantised per CTA) or, with x == nullptr, ready Q8_1 blocks in vy_in.  CTA i owns the
// contiguous rows [i * total / grid, (i + 1) * total / grid), warps take every 8th of them.
// Before waiting for the previous kernel (programmatic dependent launch) the CTA asks L2 to fetch
// its weight rows, which do not depend on that kernel.
struct MvParams {
    const uint8_t *w[3];
    int n[3];
    int k;
    const void *x;
    const uint8_t *vy_in;
    uint8_t *vy_out;  // CTA 0 stores the Q8_1 blocks here (kpad / 32 blocks) when not null
    int kpad;
    const float *residual;
    float *dst;
    uint32_t *status;  // optional: MMRS_ERR_TIMEOUT when a wait of the streaming kernel expired
    int pre;           // streaming kernel: groups requested before the dependency wait (0: default)
};

__device__ __forceinline__ void mv_prefetch_rows(const uint8_t *w, long r0, long r1, size_t row_bytes) {
    if (!w || r1 <= r0) return;
    const uint8_t *p = w + r0 * row_bytes;
    size_t bytes = (size_t)(r1 - r0) * row_bytes;
    while (bytes >= 16) {
        const uint32_t n = (uint32_t)std::min<size_t>(bytes, (size_t)1 << 20) & ~15u;
        prefetch_l2_bulk(p, n);
        p += n;
        bytes -= n;
    }
}

// Ready Q8_1 blocks (36 bytes, 4-byte aligned) into the shared activation.
__device__ __forceinline__ void mv_copy_q81(const uint8_t *__restrict__ vy, int nb, MvAct a, int tid, int nthreads) {
    for (int b = tid; b < nb; b += nthreads) {
        const uint8_t *blk = vy + (size_t)b * 36;
        a.d[b] = __half2float(*reinterpret_cast<const __half *>(blk));
        const int *s32 = reinterpret_cast<const int *>(blk + 4);
        int *d32 = reinterpret_cast<int *>(a.q + 32 * b);
#pragma unroll
        for (int i = 0; i < 8; ++i) d32[i] = s32[i];
    }
}

template <typename T>
__global__ void __launch_bounds__(kMvThreads) q8_0_matvec_kernel(const MvParams p) {
    extern __shared__ __align__(16) uint8_t mv_smem[];
    MvAct a{reinterpret_cast<int8_t *>(mv_smem), reinterpret_cast<float *>(mv_smem + p.kpad)};
    const int nb = p.k / 32;
    const int total = p.n[0] + p.n[1] + p.n[2];
    const int r0 = (int)((long)blockIdx.x * total / gridDim.x), r1 = (int)((long)(blockIdx.x + 1) * total / gridDim.x);
    const size_t row_bytes = (size_t)nb * 34;
    if (threadIdx.x == 0 && row_bytes % 16 == 0) {
        // rows of matrix m inside [r0, r1), when the matrix base allows 16-byte bulk requests
        const int e1 = p.n[0], e2 = p.n[0] + p.n[1];
        if (!((uintptr_t)p.w[0] & 15u)) mv_prefetch_rows(p.w[0], r0, std::min(r1, e1), row_bytes);
        if (p.n[1] && !((uintptr_t)p.w[1] & 15u))
            mv_prefetch_rows(p.w[1], std::max(r0, e1) - e1, std::min(r1, e2) - e1, row_bytes);
        if (p.n[2] && !((uintptr_t)p.w[2] & 15u))
            mv_prefetch_rows(p.w[2], std::max(r0, e2) - e2, r1 - e2, row_bytes);
    }
    grid_dependency_wait();
    launch_dependents();
    if (p.x) {
        mv_quantize<T>(static_cast<const T *>(p.x), p.k, p.kpad, a, blockIdx.x == 0 ? p.vy_out : nullptr, threadIdx.x,
                       blockDim.x);
    } else {
        mv_copy_q81(p.vy_in, nb, a, threadIdx.x, blockDim.x);
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int r = r0 + warp; r < r1; r += kMvThreads / 32) {
        // matrix by comparison (indexing the parameter arrays would copy them to local memory)
        const bool m0 = r < p.n[0], m1 = !m0 && r < p.n[0] + p.n[1];
        const uint8_t *wm = m0 ? p.w[0] : (m1 ? p.w[1] : p.w[2]);
        const int rl = m0 ? r : (m1 ? r - p.n[0] : r - p.n[0] - p.n[1]);
        const float v = mv_row_dot(wm + (size_t)rl * row_bytes, nb, a, lane);
        if (lane == 0) p.dst[r] = p.residual ? v + p.residual[r] : v;
    }
}
__host__ __device__ inline size_t mv_smem_bytes(int kpad) { return (size_t)kpad + (size_t)(kpad / 32) * sizeof(float); }

// ------------------------------------------------------------------------------------------
// Streaming matvec on a ready Q8_1 activation (rows of 16-byte multiple length, 16-byte aligned
// matrices): one CTA per SM owns a contiguous range of rows, cut into groups of whole rows of one
// matrix (<= 16 KB each).  A producer warp streams the groups through a ring of 12 shared-memory
// slots with bulk copies (about 180 KB per CTA for the Q / K / V projection): the
// first groups are requested before waiting for the previous kernel and the rest of the ring once
// the consumers hold their activation.  NC consumer warps load their lanes' activation blocks
// (lane + 32u) straight into registers, then take group j when j % NC is theirs and dot its rows
// out of shared memory.
// ------------------------------------------------------------------------------------------
constexpr int kMsSlots = 12;
constexpr int kMsSlotBytes = 16384;
// Slots requested before the dependency wait by default.  Everything in flight at once would queue
// the consumers' activation loads behind the whole stream (about 4 us for 27 MB) when the previous
// kernel is short; a few slots per SM already keep HBM busy meanwhile.  After a long kernel (the
// output projection after attention) the whole ring is requested early (MvParams::pre).
constexpr int kMsPre = 3;
constexpr int kMsMaxGroups = 96;

struct MsGroup {
    const uint8_t *src;
    int row0, rows;
};

constexpr int kMsActBytes = kMvMaxK / 32 * 36;  // the Q8_1 activation (at most 256 blocks)

static size_t ms_smem_bytes() {
    return (size_t)kMsSlots * kMsSlotBytes + kMsActBytes + sizeof(MsGroup) * kMsMaxGroups +
           sizeof(uint64_t) * (2 * kMsSlots + 1) + sizeof(int) * (kMsSlots + 1) + 16;
}

// One row of a group in shared memory against the register activation; lane l takes blocks
// l + 32u; the per-lane block order and the final butterfly are those of mv_row_dot.
template <int NBL, bool kFull>
__device__ __forceinline__ float ms_row_dot(const uint8_t *row, int nb, const int4 (&xa)[NBL][2],
                                            const float (&xd)[NBL], int lane) {
    uint32_t W[NBL][9];
#pragma unroll
    for (int u = 0; u < NBL; ++u) {
        const int b = lane + 32 * u;
        const uint32_t *w = reinterpret_cast<const uint32_t *>(row + ((34 * b) & ~3));
#pragma unroll
        for (int i = 0; i < 9; ++i) W[u][i] = (kFull || b < nb) ? w[i] : 0u;
    }
    float acc = 0.0f;
#pragma unroll
    for (int u = 0; u < NBL; ++u) {
        const int b = lane + 32 * u;
        if (!kFull && b >= nb) break;
        const bool odd = b & 1;
        const uint32_t sh = odd ? 32u : 16u;
        const float dw = __half2float(__ushort_as_half((unsigned short)((odd ? W[u][0] >> 16 : W[u][0]) & 0xFFFFu)));
        const int xv[8] = {xa[u][0].x, xa[u][0].y, xa[u][0].z, xa[u][0].w, xa[u][1].x, xa[u][1].y, xa[u][1].z, xa[u][1].w};
        int s0 = 0, s1 = 0;
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
            s0 = __dp4a((int)__funnelshift_rc(W[u][i], W[u][i + 1], sh), xv[i], s0);
            s1 = __dp4a((int)__funnelshift_rc(W[u][i + 1], W[u][i + 2], sh), xv[i + 1], s1);
        }
        acc += __fmul_rn(__fmul_rn((float)(s0 + s1), dw), xd[u]);
    }
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, m);
    return acc;
}

template <int NBL, int NC, bool kFull>
__global__ void __launch_bounds__(32 * (NC + 1), 1) q8_0_matvec_stream_kernel(const MvParams p) {
    extern __shared__ __align__(128) uint8_t ms_smem[];
    uint8_t *slots = ms_smem;
    uint8_t *act = ms_smem + (size_t)kMsSlots * kMsSlotBytes;
    MsGroup *groups = reinterpret_cast<MsGroup *>(act + kMsActBytes);
    uint64_t *full = reinterpret_cast<uint64_t *>(groups + kMsMaxGroups);
    uint64_t *empty = full + kMsSlots;
    uint64_t *abar = empty + kMsSlots;
    int *ngroups = reinterpret_cast<int *>(abar + 1);
    int *ticket = ngroups + 1;  // [kMsSlots]
    const int nb = p.k / 32, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // the activation by one bulk copy when its size is a multiple of 16 bytes (nb % 4 == 0) and
    // it is 16-byte aligned; otherwise each lane loads its blocks
    const bool act_bulk = (nb % 4) == 0 && !((uintptr_t)p.vy_in & 15u);
    const int total = p.n[0] + p.n[1] + p.n[2];
    const int r0 = (int)((long)blockIdx.x * total / gridDim.x), r1 = (int)((long)(blockIdx.x + 1) * total / gridDim.x);
    const size_t row_bytes = (size_t)nb * 34;
    const int per = std::max(1, (int)(kMsSlotBytes / row_bytes));
    const int pre = p.pre <= 0 ? kMsPre : (p.pre < kMsSlots ? p.pre : kMsSlots);
    const uint64_t deadline = globaltimer_ns() + 2000000000ull;
    if (threadIdx.x == NC * 32) {
        // groups: whole rows of one matrix, at most `per` of them
        const int e1 = p.n[0], e2 = p.n[0] + p.n[1];
        int ng = 0;
        for (int r = r0; r < r1 && ng < kMsMaxGroups;) {
            const int m = r < e1 ? 0 : (r < e2 ? 1 : 2);
            const int base = m == 0 ? 0 : (m == 1 ? e1 : e2), lim = m == 0 ? e1 : (m == 1 ? e2 : total);
            const int end = std::min({r + per, r1, lim});
            groups[ng].src = (m == 0 ? p.w[0] : (m == 1 ? p.w[1] : p.w[2])) + (size_t)(r - base) * row_bytes;
            groups[ng].row0 = r;
            groups[ng].rows = end - r;
            ++ng;
            r = end;
        }
        *ngroups = ng;
        for (int i = 0; i < kMsSlots; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
            ticket[i] = -1;
        }
        mbar_init(abar, 1);
        fence_mbar_init();
        for (int j = 0; j < ng && j < pre; ++j) {
            const uint32_t bytes = (uint32_t)(groups[j].rows * row_bytes);
            ticket[j] = j;
            mbar_arrive_expect_tx(&full[j], bytes);
            bulk_g2s(slots + (size_t)j * kMsSlotBytes, groups[j].src, bytes, &full[j]);
        }
    }
    __syncthreads();
    grid_dependency_wait();
    launch_dependents();
    const int ng = *ngroups;
    if (warp == NC) {  // producer: the activation, the rest of the ring once the consumers hold it, refills
        if (lane == 0 && act_bulk) {
            mbar_arrive_expect_tx(abar, (uint32_t)(nb * 36));
            bulk_g2s(act, p.vy_in, (uint32_t)(nb * 36), abar);
        }
        named_sync(2, 32 * (NC + 1));
        if (lane == 0) {
            for (int j = pre; j < ng; ++j) {
                const int st = j % kMsSlots;
                if (j >= kMsSlots && !mbar_wait_sleep(&empty[st], (uint32_t)(((j / kMsSlots) - 1) & 1), deadline)) {
                    if (p.status) atomicExch(p.status, (uint32_t)MMRS_ERR_TIMEOUT);
                    break;
                }
                const uint32_t bytes = (uint32_t)(groups[j].rows * row_bytes);
                *reinterpret_cast<volatile int *>(&ticket[st]) = j;
                mbar_arrive_expect_tx(&full[st], bytes);
                bulk_g2s(slots + (size_t)st * kMsSlotBytes, groups[j].src, bytes, &full[st]);
            }
        }
        return;
    }
    // this lane's activation blocks (lane + 32u), Q8_1 (half d, half sum, 32 int8), in registers
    int4 xa[NBL][2];
    float xd[NBL];
    if (act_bulk && !mbar_wait_sleep(abar, 0u, deadline) && lane == 0 && p.status)
        atomicExch(p.status, (uint32_t)MMRS_ERR_TIMEOUT);
    const uint8_t *asrc = act_bulk ? act : p.vy_in;
#pragma unroll
    for (int u = 0; u < NBL; ++u) {
        const int b = lane + 32 * u;
        const uint32_t *blk = reinterpret_cast<const uint32_t *>(asrc + (size_t)b * 36);
        uint32_t v[9];
#pragma unroll
        for (int i = 0; i < 9; ++i) v[i] = (kFull || b < nb) ? blk[i] : 0u;
        xd[u] = __half2float(__ushort_as_half((unsigned short)(v[0] & 0xFFFFu)));
        xa[u][0] = make_int4((int)v[1], (int)v[2], (int)v[3], (int)v[4]);
        xa[u][1] = make_int4((int)v[5], (int)v[6], (int)v[7], (int)v[8]);
    }
    named_arrive(2, 32 * (NC + 1));  // xd is in use: the loads have landed
    for (int j = warp; j < ng; j += NC) {
        const int st = j % kMsSlots;
        if (!ring_wait(full, ticket, st, j, kMsSlots, deadline)) {
            if (lane == 0 && p.status) atomicExch(p.status, (uint32_t)MMRS_ERR_TIMEOUT);
            break;
        }
        const uint8_t *g = slots + (size_t)st * kMsSlotBytes;
        const MsGroup gr = groups[j];
        for (int i = 0; i < gr.rows; ++i) {
            const float v = ms_row_dot<NBL, kFull>(g + (size_t)i * row_bytes, nb, xa, xd, lane);
            const int r = gr.row0 + i;
            if (lane == 0) p.dst[r] = p.residual ? v + p.residual[r] : v;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
    }
}

// Q8_1 blocks of num_rows rows (mmvq_gguf.cu:1137-1169): warp per 32-block.  Runs after the
// previous kernel completed (ordinary launch) and lets the next kernel, which streams weights that
// do not depend on it, start at once.
__global__ void __launch_bounds__(256) quantize_q8_1_rows_kernel(const float *__restrict__ x, uint8_t *__restrict__ vy,
                                                                 int kx, int kx_padded, int num_rows) {
    launch_dependents();
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const int nb = kx_padded / 32;
    if (warp >= nb * num_rows) return;
    const int row = warp / nb, b = warp % nb, i = b * 32 + lane;
    const float v = i < kx ? x[(long)row * kx + i] : 0.0f;
    float d, sum;
    const int8_t q = q81_lane(v, d, sum);
    uint8_t *blk = vy + ((long)row * nb + b) * 36;
    blk[4 + lane] = (uint8_t)q;
    if (lane == 0) {
        *reinterpret_cast<__half *>(blk) = __float2half_rn(d);
        *reinterpret_cast<__half *>(blk + 2) = __float2half_rn(sum);
    }
}

// Launch with the programmatic-serialization attribute: the kernel may start while the previous
// kernel of the stream finishes (it waits for it before reading the activation).
template <typename K, typename... Args>
static cudaError_t launch_pdl(K kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

static int sm_count() {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms;
}

template <int NBL, int NC, bool kFull>
static cudaError_t ms_launch(const MvParams &p, int grid, cudaStream_t s) {
    static std::once_flag once[64];
    int dev = 0;
    cudaGetDevice(&dev);
    std::call_once(once[dev & 63], [] {
        cudaFuncSetAttribute(q8_0_matvec_stream_kernel<NBL, NC, kFull>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)ms_smem_bytes());
    });
    return launch_pdl(q8_0_matvec_stream_kernel<NBL, NC, kFull>, dim3(grid), dim3(32 * (NC + 1)), ms_smem_bytes(), s, p);
}

// Blocks per lane 1..8 (k <= 8192); 16 consumer warps up to 3 blocks per lane (6 when every lane
// has all its blocks), 8 above.  The two shapes of the attention half (3 and 6 blocks, every lane
// full) take 11: with the producer that is 12 warps, 3 per scheduler, so a thread may use up to
// 168 registers instead of the 96 that 17 warps leave (the per-scheduler register file bounds
// the busiest scheduler).
template <bool kFull>
static cudaError_t ms_dispatch(const MvParams &p, int grid, cudaStream_t s) {
    switch ((p.k / 32 + 31) / 32) {
        case 1: return ms_launch<1, 16, kFull>(p, grid, s);
        case 2: return ms_launch<2, 16, kFull>(p, grid, s);
        case 3: return ms_launch<3, kFull ? 11 : 16, kFull>(p, grid, s);
        case 4: return ms_launch<4, kFull ? 16 : 8, kFull>(p, grid, s);
        case 5: return ms_launch<5, kFull ? 16 : 8, kFull>(p, grid, s);
        case 6: return ms_launch<6, kFull ? 11 : 8, kFull>(p, grid, s);
        case 7: return ms_launch<7, 8, kFull>(p, grid, s);
        default: return ms_launch<8, 8, kFull>(p, grid, s);
    }
}

template <typename T>
static int mv_launch(const MvParams &p, cudaStream_t s) {
    const int total = p.n[0] + p.n[1] + p.n[2];
    if (p.k <= 0 || p.k % 64 || p.k > kMvMaxK || p.kpad < p.k || p.kpad % 32 || total <= 0) return MMRS_ERR_ARG;
    for (int m = 0; m < 3; ++m)
        if (p.n[m] > 0 && (!p.w[m] || ((uintptr_t)p.w[m] & 3u))) return MMRS_ERR_ARG;
    const int sms = sm_count();
    const size_t row_bytes = (size_t)(p.k / 32) * 34;
    // the streaming kernel reads a ready Q8_1 activation: vy_in, or x quantised into vy_out first
    bool stream = row_bytes % 16 == 0 && row_bytes <= (size_t)kMsSlotBytes && (p.vy_in || (p.x && p.vy_out)) &&
                  (p.vy_in ? !((uintptr_t)p.vy_in & 3u) : !((uintptr_t)p.vy_out & 3u));
    for (int m = 0; m < 3; ++m) stream = stream && (p.n[m] == 0 || !((uintptr_t)p.w[m] & 15u));
    const int grid = std::min(sms, total);
    const int per = stream ? std::max(1, (int)(kMsSlotBytes / row_bytes)) : 1;
    stream = stream && (total / grid + 1 + per - 1) / per + 3 <= kMsMaxGroups;
    cudaError_t e;
    if (stream) {
        MvParams q = p;
        if (p.x) {  // activation -> Q8_1 once, then the matrices stream against it
            const int nbp = p.kpad / 32;
            quantize_q8_1_rows_kernel<<<(nbp * 32 + 255) / 256, 256, 0, s>>>(static_cast<const float *>(p.x), p.vy_out,
                                                                            p.k, p.kpad, 1);
            q.x = nullptr;
            q.vy_in = p.vy_out;
        }
        e = (p.k / 32) % 32 == 0 ? ms_dispatch<true>(q, grid, s) : ms_dispatch<false>(q, grid, s);
    } else {
        const int rows_per_cta = kMvThreads / 32;
        const int blocks = std::min((total + rows_per_cta - 1) / rows_per_cta, sms * 4);
        e = launch_pdl(q8_0_matvec_kernel<T>, dim3(blocks), dim3(kMvThreads), mv_smem_bytes(p.kpad), s, p);
    }
    return e == cudaSuccess ? MMRS_OK : MMRS_ERR_LAUNCH;
}

// ------------------------------------------------------------------------------------------
// Q / K RMSNorm to f16 (qkv_rmsnorm_f16_cuda1, mmvq_gguf.cu:838-885): CTA 0 = q, 1 = k, 2 = v
// (copy); sum of squares in a fixed order (thread-strided partials, warp tree, block tree).
// ------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) qkv_rmsnorm_f16_kernel(const float *__restrict__ src,
                                                               const float *__restrict__ qa,
                                                               const float *__restrict__ ka, __half *__restrict__ dst,
                                                               int q_rows, int k_rows, int v_rows, float eps) {
    __shared__ float ws[32];
    const int proj = blockIdx.x, tid = threadIdx.x;
    const int n = proj == 0 ? q_rows : (proj == 1 ? k_rows : v_rows);
    const int off = proj == 0 ? 0 : (proj == 1 ? q_rows : q_rows + k_rows);
    if (proj == 2) {
        for (int i = tid; i < n; i += blockDim.x) dst[off + i] = __float2half_rn(src[off + i]);
        return;
    }
    float ss = 0.0f;
    for (int i = tid; i < n; i += blockDim.x) ss = fmaf(src[off + i], src[off + i], ss);
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, m);
    if ((tid & 31) == 0) ws[tid >> 5] = ss;
    __syncthreads();
    float t = (tid & 31) < (int)(blockDim.x >> 5) ? ws[tid & 31] : 0.0f;
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) t += __shfl_xor_sync(0xffffffffu, t, m);
    const float scale = rsqrtf(__fdiv_rn(t, (float)n) + eps);
    const float *alpha = proj == 0 ? qa : ka;
    for (int i = tid; i < n; i += blockDim.x) dst[off + i] = __float2half_rn(__fmul_rn(__fmul_rn(scale, src[off + i]), alpha[i]));
}

// ------------------------------------------------------------------------------------------
// Partial rotary embedding (partial_rope_f16_cuda1, mmvq_gguf.cu:1038-1066), thread per output
// element of [Q rows | K rows]: columns >= rope_dim of a head are copied; the first half of the
// rotated columns is fma(x, c, -rn(x' * s)), the second fma(x', s, rn(x * c)) in half, c / s the
// f32 table entries rounded to half (the arithmetic of the reference kernel as compiled, written
// with explicit fma so that it does not depend on contraction).  K (and V, when given) go to
// k_out / v_out at (local / head_dim) * kv_stride + local % head_dim: kv_stride = head_dim for a
// contiguous output, the cache's per-head stride to append one position to a KV cache.
// ------------------------------------------------------------------------------------------
struct RopeParams {
    const __half *q, *k, *v;
    const float *cos, *sin;
    __half *q_out, *k_out, *v_out;
    int q_rows, k_rows, head_dim, rope_dim, position;
    long kv_stride;
};

__global__ void __launch_bounds__(256) partial_rope_kernel(const RopeParams p) {
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= p.q_rows + 2 * p.k_rows) return;
    if (idx >= p.q_rows + p.k_rows) {  // V copy (cache append only)
        if (!p.v) return;
        const int local = idx - p.q_rows - p.k_rows;
        p.v_out[(long)(local / p.head_dim) * p.kv_stride + local % p.head_dim] = p.v[local];
        return;
    }
    const bool is_q = idx < p.q_rows;
    const int local = is_q ? idx : idx - p.q_rows;
    const __half *src = is_q ? p.q : p.k;
    __half *dst = is_q ? p.q_out + local : p.k_out + (long)(local / p.head_dim) * p.kv_stride + local % p.head_dim;
    const int col = local % p.head_dim;
    if (col >= p.rope_dim) {
        *dst = src[local];
        return;
    }
    const int half_rope = p.rope_dim / 2;
    const bool first = col < half_rope;
    const int pair = first ? local + half_rope : local - half_rope;
    const int freq = first ? col : col - half_rope;
    const __half c = __float2half_rn(p.cos[p.position * half_rope + freq]);
    const __half sn = __float2half_rn(p.sin[p.position * half_rope + freq]);
    *dst = first ? __hfma(src[local], c, __hneg(__hmul_rn(src[pair], sn)))
                 : __hfma(src[pair], sn, __hmul_rn(src[local], c));
}

// ------------------------------------------------------------------------------------------
// Split-K GQA decode on the tensor cores.  CTA = (split, KV head g), 8 warps; the split's keys are
// 16-key chunks, chunk i of the split handled by warp i % 8 from stage i % 16 (two chunks in
// flight per warp).  A stage holds the chunk's K and V rows as four TMA tiles of 16 keys x 64 dims (f16,
// 128-byte rows, 128-byte swizzle: 16-byte column c of key r sits at column c ^ (r & 7)), so the
// ldmatrix reads below are free of bank conflicts.  Rows past seq_len arrive as zeros.
//   S = Q K^T: mma.m16n8k16 (f16 in, f32 accumulate) with the 6 query heads as M (rows 6-15 zero,
//   Q in registers) and 8 keys as N, K fragments by ldmatrix;
//   online softmax per head over the chunk; the probabilities, split into f16 hi + lo parts, are
//   reused in registers as the A operands of
//   O += P V: mma.m16n8k16 with keys as K and 8 dims as N, V fragments by ldmatrix.trans (the
//   reference's tensor-core kernel rounds P to f16; the split keeps about 22 bits).
// The warps' (max, sum, O) merge in shared memory into the split's partial per query head.
// Fused mode (single-token layer forward): the prologue computes the Q / K RMSNorm scales from the
// f32 projection, the group's 6 query heads normalised and rotated, and, in the split that holds
// the new position, its rotated K and its V (written to the caches, and into the stage in place of
// the row the TMA read); the last CTA of each KV head merges the splits and writes the attention
// output in f16 and as Q8_1 blocks for the output projection.
// ------------------------------------------------------------------------------------------
constexpr int kGqWarps = 8;
constexpr int kGqThreads = 32 * kGqWarps;
constexpr int kGqKeys = 16;               // keys per chunk
constexpr int kGqStages = 2 * kGqWarps;    // two chunks in flight per warp
constexpr int kGqPre = 8;                  // stages requested before the dependency wait
constexpr int kGqTile = kGqKeys * 128;  // bytes of one 16-key x 64-dim f16 tile
constexpr int kGqStageBytes = 4 * kGqTile;  // K dims 0-63 | K dims 64-127 | V dims 0-63 | V dims 64-127

struct GqSmem {
    uint8_t stage[kGqStages][kGqStageBytes];
    float wacc[kGqWarps][kAttnGroup][kAttnHeadDim];
    __half qh[kAttnGroup][kAttnHeadDim];
    __half qn[kAttnGroup][kAttnHeadDim];
    __half newk[kAttnHeadDim], newkn[kAttnHeadDim], newv[kAttnHeadDim];
    float wm[kGqWarps][8], wl[kGqWarps][8];
    float red[2][kGqWarps];
    float wts[kAttnGroup][kAttnMaxSplits];
    float den[kAttnGroup];
    uint64_t full[kGqStages];
    uint64_t cbar;  // the combining CTA's bulk read of the split records
    int last;
};
// Split record: plain mode [num_splits][query_heads][130] (max, sum, 128 values: the reference's
// layout); fused mode [kv_heads][num_splits][6][132] (max, sum, 2 pad, 128 values), so that one
// KV head's records are one contiguous, 16-byte aligned range for the combining CTA.
constexpr int kGqRec = 132;
constexpr int kGqMaxFusedSplits = kGqStages * kGqStageBytes / (kAttnGroup * kGqRec * 4);  // records fit the stages
static_assert(kGqThreads == 2 * kAttnHeadDim && (kAttnGroup * kAttnHeadDim) % kGqThreads == 0,
              "the prologue and the split merge assume 256 threads");
constexpr size_t kGqSmemBytes = sizeof(GqSmem) + 1024;  // + alignment of the swizzled stages

struct GqaParams {
    // plain mode: q f16 [query_heads][q_head_stride] (normalised and rotated already)
    const __half *q;
    int q_head_stride;
    // fused mode
    const float *proj;  // f32 [q_rows + 2 k_rows] = [Wq x | Wk x | Wv x]
    const float *q_norm, *k_norm, *cos, *sin;
    float eps;
    int rope_dim;
    __half *k_cache, *v_cache;  // append target: head g at g * cache_head_stride, position at + pos * 128
    long cache_head_stride;
    uint32_t *tickets;  // [kv_heads], zero before first use, left zero
    uint32_t *status;   // MMRS_ERR_TIMEOUT when a wait expired
    __half *out;        // fused: attention output f16 [query_heads][128]
    uint8_t *vy;        // fused: the same as Q8_1 blocks [query_heads * 4]
    float *partials;    // [num_splits][query_heads][130]
    int seq_len, num_splits, query_heads;
    float scale;
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr)
                 : "memory");
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr)
                 : "memory");
}
// D = A B + D, m16n8k16, A rows 8-15 zero (a1 = a3 = 0): only d0, d1 (row lane / 4) are carried.
__device__ __forceinline__ void mma_rows8(float &d0, float &d1, uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
    float e2 = 0.0f, e3 = 0.0f;
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d0), "+f"(d1), "+f"(e2), "+f"(e3)
        : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&h);
}
// Byte offset of 16-byte column c (0-15 over the 128 dims) of key r inside a K or V stage half.
__device__ __forceinline__ uint32_t gq_swz(int r, int c) {
    return (uint32_t)((c >> 3) * kGqTile + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

template <bool kFused>
__global__ void __launch_bounds__(kGqThreads, 1)
    gqa_tc_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                  const GqaParams p) {
    extern __shared__ uint8_t gq_raw[];
    GqSmem &sm = *reinterpret_cast<GqSmem *>((reinterpret_cast<uintptr_t>(gq_raw) + 1023) & ~uintptr_t(1023));
    const int split = blockIdx.x, g = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int seq = p.seq_len, pos = seq - 1;
    const int nch = (seq + kGqKeys - 1) / kGqKeys;
    const int c0 = (int)((long)split * nch / p.num_splits), c1 = (int)((long)(split + 1) * nch / p.num_splits);
    const int mine = c1 - c0;
    const bool holds_pos = kFused && pos / kGqKeys >= c0 && pos / kGqKeys < c1;
    auto issue = [&](int i) {
        const int st = i % kGqStages, key0 = (c0 + i) * kGqKeys;
        uint8_t *dst = sm.stage[st];
        mbar_arrive_expect_tx(&sm.full[st], kGqStageBytes);
        tma_load_3d(dst, &kmap, 0, key0, g, &sm.full[st]);
        tma_load_3d(dst + kGqTile, &kmap, 64, key0, g, &sm.full[st]);
        tma_load_3d(dst + 2 * kGqTile, &vmap, 0, key0, g, &sm.full[st]);
        tma_load_3d(dst + 3 * kGqTile, &vmap, 64, key0, g, &sm.full[st]);
    };
    if (tid == 0) {
        for (int i = 0; i < kGqStages; ++i) mbar_init(&sm.full[i], 1);
        mbar_init(&sm.cbar, 1);
        fence_mbar_init();
        // the cached keys come from earlier launches: the first loads start before the wait below,
        // the rest once the prologue's own loads have landed (so they do not queue behind them)
        for (int i = 0; i < mine && i < kGqPre; ++i) issue(i);
    }
    grid_dependency_wait();
    launch_dependents();
    if constexpr (kFused) {
        // every global value the prologue needs is requested before any arithmetic: the Q and K
        // rows for the RMSNorm sums (q_rows <= 8192: at most 8 float4 per thread), the group's
        // 6 heads with their norm weights and rotary entries (3 values per thread), and head g's
        // K / V row (threads 0-127)
        const int qr = p.query_heads * kAttnHeadDim, kr = qr / kAttnGroup, half_rope = p.rope_dim / 2;
        const float4 *p4 = reinterpret_cast<const float4 *>(p.proj);
        constexpr int kQ4 = kMvMaxK / 4 / kGqThreads, kK4 = (kMvMaxK / kAttnGroup / 4 + kGqThreads - 1) / kGqThreads;
        constexpr int kQe = kAttnGroup * kAttnHeadDim / kGqThreads;
        float4 vq[kQ4], vk[kK4];
#pragma unroll
        for (int u = 0; u < kQ4; ++u) {
            const int i = tid + u * kGqThreads;
            vq[u] = i < qr / 4 ? p4[i] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
#pragma unroll
        for (int u = 0; u < kK4; ++u) {
            const int i = tid + u * kGqThreads;
            vk[u] = i < kr / 4 ? p4[qr / 4 + i] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
        float pq[kQe], aq[kQe], cq6[kQe], sq6[kQe];
#pragma unroll
        for (int u = 0; u < kQe; ++u) {
            const int e = tid + u * kGqThreads, col = e % kAttnHeadDim;
            const int qi = g * kAttnGroup * kAttnHeadDim + e;
            pq[u] = p.proj[qi];
            aq[u] = p.q_norm[qi];
            const int freq = col < half_rope ? col : col - half_rope;
            const bool rot = col < p.rope_dim;
            cq6[u] = rot ? p.cos[(long)pos * half_rope + freq] : 0.0f;
            sq6[u] = rot ? p.sin[(long)pos * half_rope + freq] : 0.0f;
        }
        float pk = 0.0f, ak = 0.0f, pv = 0.0f, ck = 0.0f, sk1 = 0.0f;
        const bool krow = holds_pos && tid < kAttnHeadDim;
        if (krow) {
            const int ki = g * kAttnHeadDim + tid, freq = tid < half_rope ? tid : tid - half_rope;
            pk = p.proj[qr + ki];
            ak = p.k_norm[ki];
            pv = p.proj[qr + kr + ki];
            if (tid < p.rope_dim) {
                ck = p.cos[(long)pos * half_rope + freq];
                sk1 = p.sin[(long)pos * half_rope + freq];
            }
        }
        // RMSNorm scales of all Q rows and all K rows (fixed order: per-thread chain, butterfly, warps)
        float sq = 0.0f, sk = 0.0f;
#pragma unroll
        for (int u = 0; u < kQ4; ++u) {
            sq = fmaf(vq[u].x, vq[u].x, sq);
            sq = fmaf(vq[u].y, vq[u].y, sq);
            sq = fmaf(vq[u].z, vq[u].z, sq);
            sq = fmaf(vq[u].w, vq[u].w, sq);
        }
#pragma unroll
        for (int u = 0; u < kK4; ++u) {
            sk = fmaf(vk[u].x, vk[u].x, sk);
            sk = fmaf(vk[u].y, vk[u].y, sk);
            sk = fmaf(vk[u].z, vk[u].z, sk);
            sk = fmaf(vk[u].w, vk[u].w, sk);
        }
#pragma unroll
        for (int m = 16; m > 0; m >>= 1) {
            sq += __shfl_xor_sync(0xffffffffu, sq, m);
            sk += __shfl_xor_sync(0xffffffffu, sk, m);
        }
        if (lane == 0) {
            sm.red[0][warp] = sq;
            sm.red[1][warp] = sk;
        }
        __syncthreads();
        if (tid == 0)
            for (int i = kGqPre; i < mine && i < kGqStages; ++i) issue(i);
        float tq = 0.0f, tk = 0.0f;
#pragma unroll
        for (int w = 0; w < kGqWarps; ++w) {
            tq += sm.red[0][w];
            tk += sm.red[1][w];
        }
        const float scq = rsqrtf(__fdiv_rn(tq, (float)qr) + p.eps), sck = rsqrtf(__fdiv_rn(tk, (float)kr) + p.eps);
        // qkv_rmsnorm_f16: f16(scale * v * alpha) for the group's 6 heads (and head g of K, V)
#pragma unroll
        for (int u = 0; u < kQe; ++u)
            (&sm.qn[0][0])[tid + u * kGqThreads] = __float2half_rn(__fmul_rn(__fmul_rn(scq, pq[u]), aq[u]));
        if (krow) {
            sm.newkn[tid] = __float2half_rn(__fmul_rn(__fmul_rn(sck, pk), ak));
            sm.newv[tid] = __float2half_rn(pv);
        }
        __syncthreads();
        // RoPE (partial_rope_kernel arithmetic) with the rotary entries already in registers
#pragma unroll
        for (int u = 0; u < kQe; ++u) {
            const int e = tid + u * kGqThreads, h = e / kAttnHeadDim, col = e % kAttnHeadDim;
            __half r = sm.qn[h][col];
            if (col < p.rope_dim) {
                const bool first = col < half_rope;
                const __half c = __float2half_rn(cq6[u]), sn = __float2half_rn(sq6[u]);
                const __half x = sm.qn[h][col], xp = sm.qn[h][first ? col + half_rope : col - half_rope];
                r = first ? __hfma(x, c, __hneg(__hmul_rn(xp, sn))) : __hfma(xp, sn, __hmul_rn(x, c));
            }
            sm.qh[h][col] = r;
        }
        if (krow) {
            __half kv = sm.newkn[tid];
            if (tid < p.rope_dim) {
                const bool first = tid < half_rope;
                const __half c = __float2half_rn(ck), sn = __float2half_rn(sk1);
                const __half x = sm.newkn[tid], xp = sm.newkn[first ? tid + half_rope : tid - half_rope];
                kv = first ? __hfma(x, c, __hneg(__hmul_rn(xp, sn))) : __hfma(xp, sn, __hmul_rn(x, c));
            }
            sm.newk[tid] = kv;
            const long at = (long)g * p.cache_head_stride + (long)pos * kAttnHeadDim + tid;
            p.k_cache[at] = kv;
            p.v_cache[at] = sm.newv[tid];
        }
    } else {
        for (int e = tid; e < kAttnGroup * kAttnHeadDim; e += kGqThreads) {
            const int h = e / kAttnHeadDim, col = e % kAttnHeadDim;
            sm.qh[h][col] = p.q[(long)(g * kAttnGroup + h) * p.q_head_stride + col];
        }
        __syncthreads();
        if (tid == 0)
            for (int i = kGqPre; i < mine && i < kGqStages; ++i) issue(i);
    }
    __syncthreads();
    // Q as the A operand: row lane / 4 (query head of the group; rows 6-15 zero), dims of k-step s
    const int gq = lane >> 2, cq = 2 * (lane & 3);
    uint32_t qa0[8], qa2[8];
#pragma unroll
    for (int s8 = 0; s8 < 8; ++s8) {
        qa0[s8] = gq < kAttnGroup ? *reinterpret_cast<const uint32_t *>(&sm.qh[gq][16 * s8 + cq]) : 0u;
        qa2[s8] = gq < kAttnGroup ? *reinterpret_cast<const uint32_t *>(&sm.qh[gq][16 * s8 + 8 + cq]) : 0u;
    }
    float m_run = -INFINITY, l_run = 0.0f;
    float o[16][2];
#pragma unroll
    for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = 0.0f;
    const uint64_t deadline = globaltimer_ns() + 2000000000ull;
    bool ok = true;
    for (int i = warp; i < mine; i += kGqWarps) {
        const int st = i % kGqStages;
        if (!mbar_wait_sleep(&sm.full[st], (uint32_t)((i / kGqStages) & 1), deadline)) {
            ok = false;
            break;
        }
        uint8_t *sb = sm.stage[st];
        const int key0 = (c0 + i) * kGqKeys, nvalid = min(kGqKeys, seq - key0);
        if (kFused && pos >= key0 && pos < key0 + kGqKeys) {  // the new position replaces the cached row
            const uint32_t off = gq_swz(pos - key0, lane >> 1) + (lane & 1) * 8;
            *reinterpret_cast<uint2 *>(sb + off) = *reinterpret_cast<const uint2 *>(&sm.newk[4 * lane]);
            *reinterpret_cast<uint2 *>(sb + 2 * kGqTile + off) = *reinterpret_cast<const uint2 *>(&sm.newv[4 * lane]);
            __syncwarp();
        }
        const uint32_t sbase = smem_u32(sb);
        // S = Q K^T: n-tile t = keys 8t..8t+7; the lane holds head gq, keys 8t + cq + {0, 1}
        constexpr int NT = kGqKeys / 8;  // n-tiles of 8 keys
        float sc[NT][2];
#pragma unroll
        for (int t = 0; t < NT; ++t) sc[t][0] = sc[t][1] = 0.0f;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {  // k-steps 2kk, 2kk + 1 of the four n-tiles, independent mmas adjacent
            uint32_t b[NT][4];
#pragma unroll
            for (int t = 0; t < NT; ++t)
                ldsm_x4(sbase + gq_swz(8 * t + (lane & 7), 4 * kk + (lane >> 3)), b[t][0], b[t][1], b[t][2], b[t][3]);
#pragma unroll
            for (int t = 0; t < NT; ++t) mma_rows8(sc[t][0], sc[t][1], qa0[2 * kk], qa2[2 * kk], b[t][0], b[t][1]);
#pragma unroll
            for (int t = 0; t < NT; ++t)
                mma_rows8(sc[t][0], sc[t][1], qa0[2 * kk + 1], qa2[2 * kk + 1], b[t][2], b[t][3]);
        }
        // online softmax of head gq over the chunk (its 16 keys sit on the 4 lanes of the quad)
        float mx = -INFINITY;
#pragma unroll
        for (int t = 0; t < NT; ++t)
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                const float v = 8 * t + cq + c < nvalid ? sc[t][c] * p.scale : -INFINITY;
                sc[t][c] = v;
                mx = fmaxf(mx, v);
            }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float mn = fmaxf(m_run, mx);  // finite: key 0 of every chunk is valid
        const float alpha = m_run == -INFINITY ? 0.0f : expf(m_run - mn);
        // probabilities as f16 pairs hi + lo (hi = f16(p), lo = f16(p - hi)): two tensor-core
        // products carry p to about 22 bits
        uint32_t pa[NT], pb[NT];
        float ps = 0.0f;
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            const float p0 = expf(sc[t][0] - mn), p1 = expf(sc[t][1] - mn);
            const __half2 ph = __floats2half2_rn(p0, p1);
            const float2 pf = __half22float2(ph);
            const __half2 pl = __floats2half2_rn(p0 - pf.x, p1 - pf.y);
            pa[t] = *reinterpret_cast<const uint32_t *>(&ph);
            pb[t] = *reinterpret_cast<const uint32_t *>(&pl);
            ps += p0 + p1;
        }
        ps += __shfl_xor_sync(0xffffffffu, ps, 1);
        ps += __shfl_xor_sync(0xffffffffu, ps, 2);
        l_run = fmaf(l_run, alpha, ps);
        m_run = mn;
#pragma unroll
        for (int n = 0; n < 16; ++n) {
            o[n][0] *= alpha;
            o[n][1] *= alpha;
        }
        // O += P V: k-step j = keys 16j..16j+15 (A = probabilities of n-tiles 2j, 2j + 1), n-tile = 8 dims
#pragma unroll
        for (int j = 0; j < NT / 2; ++j) {
            const int r = 16 * j + ((lane >> 3) & 1) * 8 + (lane & 7);
            uint32_t b[8][4];
#pragma unroll
            for (int dp = 0; dp < 8; ++dp)
                ldsm_x4_t(sbase + 2 * kGqTile + gq_swz(r, 2 * dp + (lane >> 4)), b[dp][0], b[dp][1], b[dp][2], b[dp][3]);
#pragma unroll
            for (int n = 0; n < 16; ++n)
                mma_rows8(o[n][0], o[n][1], pa[2 * j], pa[2 * j + 1], b[n >> 1][2 * (n & 1)], b[n >> 1][2 * (n & 1) + 1]);
#pragma unroll
            for (int n = 0; n < 16; ++n)
                mma_rows8(o[n][0], o[n][1], pb[2 * j], pb[2 * j + 1], b[n >> 1][2 * (n & 1)], b[n >> 1][2 * (n & 1) + 1]);
        }
        __syncwarp();
        if (i + kGqStages < mine && lane == 0) {  // refill the stage this warp just read
            fence_proxy_async_smem();
            issue(i + kGqStages);
        }
    }
    if (!ok && p.status) atomicExch(p.status, (uint32_t)MMRS_ERR_TIMEOUT);
    // merge the 4 warps: each publishes (m, l, O), thread d combines dim d of every head
    if ((lane & 3) == 0 && gq < kAttnGroup) {
        sm.wm[warp][gq] = m_run;
        sm.wl[warp][gq] = l_run;
    }
    if (gq < kAttnGroup) {
#pragma unroll
        for (int n = 0; n < 16; ++n)
            *reinterpret_cast<float2 *>(&sm.wacc[warp][gq][8 * n + cq]) = make_float2(o[n][0], o[n][1]);
    }
    __syncthreads();
    {
        const int d = tid % kAttnHeadDim, h0 = tid / kAttnHeadDim * (kAttnGroup / 2);  // 256 threads: 2 x 3 heads
#pragma unroll
        for (int h = h0; h < h0 + kAttnGroup / 2; ++h) {
            float M = -INFINITY;
#pragma unroll
            for (int w = 0; w < kGqWarps; ++w) M = fmaxf(M, sm.wm[w][h]);
            float L = 0.0f, A = 0.0f;
            if (M != -INFINITY) {
#pragma unroll
                for (int w = 0; w < kGqWarps; ++w) {
                    if (sm.wm[w][h] == -INFINITY) continue;
                    const float e = expf(sm.wm[w][h] - M);
                    L = fmaf(sm.wl[w][h], e, L);
                    A = fmaf(sm.wacc[w][h][d], e, A);
                }
            }
            float *rec = kFused ? p.partials + ((long)(g * p.num_splits + split) * kAttnGroup + h) * kGqRec
                                : p.partials + ((long)split * p.query_heads + g * kAttnGroup + h) * kAttnPartial;
            if (d == 0) {
                rec[0] = M == -INFINITY ? -FLT_MAX : M;
                rec[1] = L;
            }
            rec[(kFused ? 4 : 2) + d] = A;
        }
    }
    if constexpr (kFused) {
        // the last CTA of KV head g merges the splits (gqa_combine_f16_128 arithmetic)
        __syncthreads();
        if (tid == 0) {
            __threadfence();
            sm.last = atomicAdd(&p.tickets[g], 1u) == (uint32_t)(p.num_splits - 1);
        }
        __syncthreads();
        if (!sm.last) return;
        __threadfence();
        // the bulk read below sees the other CTAs' records and follows this CTA's reads of the stages
        asm volatile("fence.proxy.async;" ::: "memory");
        const int S = p.num_splits;
        const float *cs = reinterpret_cast<const float *>(sm.stage[0]);
        if (tid == 0) {
            p.tickets[g] = 0u;
            const uint32_t bytes = (uint32_t)(S * kAttnGroup * kGqRec * 4);
            mbar_arrive_expect_tx(&sm.cbar, bytes);
            bulk_g2s(sm.stage[0], p.partials + (long)g * S * kAttnGroup * kGqRec, bytes, &sm.cbar);
        }
        if (!mbar_wait_sleep(&sm.cbar, 0u, deadline)) {
            if (tid == 0 && p.status) atomicExch(p.status, (uint32_t)MMRS_ERR_TIMEOUT);
            return;
        }
        // weights exp(max_s - max) of the splits with a non-zero sum, and the denominator, per head
        for (int h = warp; h < kAttnGroup; h += kGqWarps) {
            float M = -FLT_MAX;
            for (int s2 = lane; s2 < S; s2 += 32) M = fmaxf(M, cs[(s2 * kAttnGroup + h) * kGqRec]);
#pragma unroll
            for (int m = 16; m > 0; m >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, m));
            float den = 0.0f;
            for (int s2 = lane; s2 < S; s2 += 32) {
                const float *rec = cs + (s2 * kAttnGroup + h) * kGqRec;
                const float w = rec[1] == 0.0f ? 0.0f : expf(rec[0] - M);
                sm.wts[h][s2] = w;
                den = fmaf(rec[1], w, den);
            }
#pragma unroll
            for (int m = 16; m > 0; m >>= 1) den += __shfl_xor_sync(0xffffffffu, den, m);
            if (lane == 0) sm.den[h] = den;
        }
        __syncthreads();
        // 6 heads x 32 four-dim items over 128 threads (warps 0-1 take a second item)
        for (int idx = tid; idx < kAttnGroup * 32; idx += kGqThreads) {
            const int h = idx >> 5, d4 = idx & 31, qh = g * kAttnGroup + h;
            float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            for (int s2 = 0; s2 < S; ++s2) {
                const float4 v = reinterpret_cast<const float4 *>(cs + (s2 * kAttnGroup + h) * kGqRec + 4)[d4];
                const float w = sm.wts[h][s2];
                acc.x = fmaf(v.x, w, acc.x);
                acc.y = fmaf(v.y, w, acc.y);
                acc.z = fmaf(v.z, w, acc.z);
                acc.w = fmaf(v.w, w, acc.w);
            }
            const float dn = sm.den[h];
            const __half2 h01 = __floats2half2_rn(__fdiv_rn(acc.x, dn), __fdiv_rn(acc.y, dn));
            const __half2 h23 = __floats2half2_rn(__fdiv_rn(acc.z, dn), __fdiv_rn(acc.w, dn));
            const long e = (long)qh * kAttnHeadDim + 4 * d4;
            uint2 packed_h;
            packed_h.x = *reinterpret_cast<const uint32_t *>(&h01);
            packed_h.y = *reinterpret_cast<const uint32_t *>(&h23);
            *reinterpret_cast<uint2 *>(p.out + e) = packed_h;
            // Q8_1 of the f16 output for the output projection: 8 lanes hold one 32-block; amax / d /
            // q as quantize_q8_1, the sum in the order of its lane-0 butterfly
            const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
            float v[4] = {f01.x, f01.y, f23.x, f23.y};
            float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
            float sm4[4] = {v[0], v[1], v[2], v[3]};
#pragma unroll
            for (int m = 4; m > 0; m >>= 1) {
                amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, m));
#pragma unroll
                for (int c = 0; c < 4; ++c) sm4[c] += __shfl_xor_sync(0xffffffffu, sm4[c], m);
            }
            sm4[0] += sm4[2];
            sm4[1] += sm4[3];
            sm4[0] += sm4[1];
            const float d = __fdiv_rn(amax, 127.0f);
            uint32_t packed = 0;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int q = amax == 0.0f ? 0 : (int)roundf(__fdiv_rn(v[c], d));
                packed |= (uint32_t)(q & 0xFF) << (8 * c);
            }
            uint8_t *blk = p.vy + (e / 32) * 36;
            *reinterpret_cast<uint32_t *>(blk + 4 + (e % 32)) = packed;
            if ((d4 & 7) == 0)
                *reinterpret_cast<uint32_t *>(blk) = (uint32_t)__half_as_ushort(__float2half_rn(d)) |
                                                     ((uint32_t)__half_as_ushort(__float2half_rn(sm4[0])) << 16);
        }
    }
}

// Merge of the splits (gqa_combine_f16_128, decode_attention.cu:791-843): weights
// exp(max_s - max) for splits with a non-zero sum, output = sum_s w_s v_s / sum_s w_s l_s.
__global__ void __launch_bounds__(128) gqa_combine_kernel(const float *__restrict__ partials, __half *__restrict__ out,
                                                          int num_splits, int query_heads) {
    __shared__ float wts[kAttnMaxSplits];
    __shared__ float den;
    const int qh = blockIdx.x, d = threadIdx.x;
    const float *base = partials + (long)qh * kAttnPartial;
    const long stride = (long)query_heads * kAttnPartial;
    float M = -FLT_MAX;
    for (int s = 0; s < num_splits; ++s) M = fmaxf(M, base[s * stride]);
    if (d < num_splits) {
        const float *rec = base + d * stride;
        wts[d] = rec[1] == 0.0f ? 0.0f : expf(rec[0] - M);
    }
    __syncthreads();
    if (d == 0) {
        float t = 0.0f;
        for (int s = 0; s < num_splits; ++s) t = fmaf(base[s * stride + 1], wts[s], t);
        den = t;
    }
    __syncthreads();
    float v = 0.0f;
    for (int s = 0; s < num_splits; ++s) v = fmaf(base[s * stride + 2 + d], wts[s], v);
    out[(long)qh * kAttnHeadDim + d] = __float2half_rn(__fdiv_rn(v, den));
}


static int rope_launch(const RopeParams &r, cudaStream_t s) {
    if (r.q_rows < 0 || r.k_rows < 0 || r.head_dim <= 0 || r.rope_dim < 0 || r.rope_dim > r.head_dim ||
        r.rope_dim % 2 || r.position < 0 || (r.q_rows && !r.q) || (r.k_rows && !r.k) || (r.rope_dim && (!r.cos || !r.sin)))
        return MMRS_ERR_ARG;
    const int total = r.q_rows + (r.v ? 2 : 1) * r.k_rows;
    if (total == 0) return MMRS_OK;
    partial_rope_kernel<<<(total + 255) / 256, 256, 0, s>>>(r);
    return cudaGetLastError() == cudaSuccess ? MMRS_OK : MMRS_ERR_LAUNCH;
}

// Tensor map over an f16 KV cache: [heads][rows][128], head h at h * head_stride elements; box =
// 64 dims x 16 positions of one head, 128-byte swizzle; rows past `rows` read as zeros.
static int make_kv_map(CUtensorMap *map, const void *base, int rows, int heads, long head_stride) {
    auto enc = tensor_map_encoder();
    if (!enc) return MMRS_ERR_LAUNCH;
    cuuint64_t dims[3] = {(cuuint64_t)kAttnHeadDim, (cuuint64_t)rows, (cuuint64_t)heads};
    cuuint64_t strides[2] = {(cuuint64_t)kAttnHeadDim * 2, (cuuint64_t)head_stride * 2};
    cuuint32_t box[3] = {64, (cuuint32_t)kGqKeys, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void *>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? MMRS_OK : MMRS_ERR_ARG;
}

static void gqa_smem_setup() {
    static std::once_flag once[64];
    int dev = 0;
    cudaGetDevice(&dev);
    std::call_once(once[dev & 63], [] {
        cudaFuncSetAttribute(gqa_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGqSmemBytes);
        cudaFuncSetAttribute(gqa_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGqSmemBytes);
    });
}

// Plain mode (launch_gqa_decode_mma_f16_128): the split kernel, then the combine kernel.
static int gqa_launch(const GqaParams &g, int kv_heads, const __half *k, const __half *v, long k_head_stride,
                      long v_head_stride, __half *out, cudaStream_t s) {
    if (!g.q || !k || !v || !g.partials || !out || g.seq_len < 1 || g.num_splits < 1 ||
        g.num_splits > kAttnMaxSplits || kv_heads < 1 || g.query_heads != kAttnGroup * kv_heads ||
        g.q_head_stride < kAttnHeadDim || k_head_stride < (long)g.seq_len * kAttnHeadDim ||
        v_head_stride < (long)g.seq_len * kAttnHeadDim || ((uintptr_t)k & 15u) || ((uintptr_t)v & 15u) ||
        (k_head_stride % 8) || (v_head_stride % 8) || ((uintptr_t)g.q & 3u) || (g.q_head_stride % 2))
        return MMRS_ERR_ARG;
    CUtensorMap kmap, vmap;
    int rc = make_kv_map(&kmap, k, g.seq_len, kv_heads, k_head_stride);
    if (rc == MMRS_OK) rc = make_kv_map(&vmap, v, g.seq_len, kv_heads, v_head_stride);
    if (rc != MMRS_OK) return rc;
    gqa_smem_setup();
    if (launch_pdl(gqa_tc_kernel<false>, dim3(g.num_splits, kv_heads), dim3(kGqThreads), kGqSmemBytes, s, kmap, vmap,
                   g) != cudaSuccess)
        return MMRS_ERR_LAUNCH;
    gqa_combine_kernel<<<g.query_heads, 128, 0, s>>>(g.partials, out, g.num_splits, g.query_heads);
    return cudaGetLastError() == cudaSuccess ? MMRS_OK : MMRS_ERR_LAUNCH;
}

static int qkv_launch(const void *x, void *vy, const void *vq, const void *vk, const void *vv, float *proj, int kx,
                      int kx_padded, int q_rows, int k_rows, int v_rows, cudaStream_t s, uint32_t *status = nullptr) {
    if (!x || q_rows < 0 || k_rows < 0 || v_rows < 0) return MMRS_ERR_ARG;
    MvParams p = {};
    p.w[0] = static_cast<const uint8_t *>(vq);
    p.w[1] = static_cast<const uint8_t *>(vk);
    p.w[2] = static_cast<const uint8_t *>(vv);
    p.n[0] = q_rows;
    p.n[1] = k_rows;
    p.n[2] = v_rows;
    p.k = kx;
    p.kpad = kx_padded;
    p.x = x;
    p.vy_out = static_cast<uint8_t *>(vy);
    p.dst = proj;
    p.status = status;
    return mv_launch<float>(p, s);
}

// Row RMSNorm of the hidden state (candle-nn RmsNorm, src/model.rs:198-210: attn_norm / ffn_norm):
// y = x / sqrt(mean(x^2) + eps) * w, one CTA per row, fixed reduction order.
__global__ void __launch_bounds__(1024) rmsnorm_rows_kernel(const float *__restrict__ x, const float *__restrict__ w,
                                                            float *__restrict__ y, int n, float eps) {
    __shared__ float ws[32];
    const float *xr = x + (long)blockIdx.x * n;
    float *yr = y + (long)blockIdx.x * n;
    float ss = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) ss = fmaf(xr[i], xr[i], ss);
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, m);
    if ((threadIdx.x & 31) == 0) ws[threadIdx.x >> 5] = ss;
    __syncthreads();
    float t = (int)(threadIdx.x & 31) < (int)(blockDim.x >> 5) ? ws[threadIdx.x & 31] : 0.0f;
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) t += __shfl_xor_sync(0xffffffffu, t, m);
    const float scale = rsqrtf(__fdiv_rn(t, (float)n) + eps);
    for (int i = threadIdx.x; i < n; i += blockDim.x) yr[i] = __fmul_rn(__fmul_rn(xr[i], scale), w[i]);
}

}  // namespace mmrs

using namespace mmrs;

extern "C" int mmrs_rmsnorm_f32(const float *x, const float *weight, float *y, int n, int rows, float eps,
                                mmrs_stream_t stream) {
    if (!x || !weight || !y || n <= 0 || rows <= 0) return MMRS_ERR_ARG;
    rmsnorm_rows_kernel<<<rows, 1024, 0, (cudaStream_t)stream>>>(x, weight, y, n, eps);
    return cudaGetLastError() == cudaSuccess ? MMRS_OK : MMRS_ERR_LAUNCH;
}

// ------------------------------------------------------------------------------------------
// C ABI
// ------------------------------------------------------------------------------------------
extern "C" void launch_mmvq_gguf_quantize_q8_1_f32(const void *x, void *vy, int kx, int kx_padded, int num_rows,
                                                   void *stream) {
    if (!x || !vy || kx <= 0 || kx_padded < kx || kx_padded % 32 || num_rows <= 0) {
        record_error(MMRS_ERR_ARG);
        return;
    }
    const long warps = (long)(kx_padded / 32) * num_rows;
    quantize_q8_1_rows_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
        static_cast<const float *>(x), static_cast<uint8_t *>(vy), kx, kx_padded, num_rows);
    record_error(cudaGetLastError() == cudaSuccess ? MMRS_OK : MMRS_ERR_LAUNCH);
}

extern "C" void launch_mmvq_gguf_q8_0_f32_plain(const void *vx, const void *vy, void *dst, int ncols_x, int nrows_x,
                                                int stride_col_y, int stride_col_dst, int b_size, void *stream) {
    (void)stride_col_dst;  // one column: its stride does not matter
    if (b_size != 1) {
        record_error(MMRS_ERR_UNSUPPORTED);
        return;
    }
    if (!vx || !vy || !dst || nrows_x <= 0 || stride_col_y * 32 < ncols_x) {
        record_error(MMRS_ERR_ARG);
        return;
    }
    MvParams p = {};
    p.w[0] = static_cast<const uint8_t *>(vx);
    p.n[0] = nrows_x;
    p.k = ncols_x;
    p.kpad = stride_col_y * 32;
    p.vy_in = static_cast<const uint8_t *>(vy);
    p.dst = static_cast<float *>(dst);
    record_error(mv_launch<float>(p, (cudaStream_t)stream));
}

extern "C" void launch_mmvq_gguf_qkv_q8_0_f32(const void *x, void *vy, const void *vq, const void *vk, const void *vv,
                                             void *dst, int kx, int kx_padded, int q_rows, int k_rows, int v_rows,
                                             void *stream) {
    record_error(qkv_launch(x, vy, vq, vk, vv, static_cast<float *>(dst), kx, kx_padded, q_rows, k_rows, v_rows,
                            (cudaStream_t)stream));
}

extern "C" void launch_mmvq_gguf_qkv_q8_0_f32_rmsnorm_f16(const void *x, void *vy, const void *vq, const void *vk,
                                                         const void *vv, void *projection_dst, const void *q_alpha,
                                                         const void *k_alpha, void *dst, int kx, int kx_padded,
                                                         int q_rows, int k_rows, int v_rows, float eps, void *stream) {
    cudaStream_t s = (cudaStream_t)stream;
    if (!projection_dst || !dst || !q_alpha || !k_alpha) {
        record_error(MMRS_ERR_ARG);
        return;
    }
    int rc = qkv_launch(x, vy, vq, vk, vv, static_cast<float *>(projection_dst), kx, kx_padded, q_rows, k_rows,
                        v_rows, s);
    if (rc == MMRS_OK) {
        qkv_rmsnorm_f16_kernel<<<3, 1024, 0, s>>>(static_cast<const float *>(projection_dst),
                                                  static_cast<const float *>(q_alpha),
                                                  static_cast<const float *>(k_alpha), static_cast<__half *>(dst),
                                                  q_rows, k_rows, v_rows, eps);
        rc = cudaGetLastError() == cudaSuccess ? MMRS_OK : MMRS_ERR_LAUNCH;
    }
    record_error(rc);
}

extern "C" void launch_partial_rope_f16(const void *q, const void *k, const void *cos, const void *sin, void *dst,
                                        int q_rows, int k_rows, int head_dim, int rope_dim, int position,
                                        void *stream) {
    if (!dst) {
        record_error(MMRS_ERR_ARG);
        return;
    }
    RopeParams r = {};
    r.q = static_cast<const __half *>(q);
    r.k = static_cast<const __half *>(k);
    r.cos = static_cast<const float *>(cos);
    r.sin = static_cast<const float *>(sin);
    r.q_out = static_cast<__half *>(dst);
    r.k_out = static_cast<__half *>(dst) + q_rows;
    r.q_rows = q_rows;
    r.k_rows = k_rows;
    r.head_dim = head_dim;
    r.rope_dim = rope_dim;
    r.position = position;
    r.kv_stride = head_dim;
    record_error(rope_launch(r, (cudaStream_t)stream));
}

extern "C" void launch_gqa_decode_mma_f16_128(const void *q, const void *k, const void *v, void *partials,
                                              void *output, int seq_len, int q_head_stride, int k_head_stride,
                                              int v_head_stride, int num_splits, int query_heads, int kv_heads,
                                              float scale, int device_ordinal, void *stream) {
    (void)device_ordinal;  // no per-device kernel configuration is needed here
    GqaParams g = {};
    g.q = static_cast<const __half *>(q);
    g.q_head_stride = q_head_stride;
    g.partials = static_cast<float *>(partials);
    g.seq_len = seq_len;
    g.num_splits = num_splits;
    g.query_heads = query_heads;
    g.scale = scale;
    record_error(gqa_launch(g, kv_heads, static_cast<const __half *>(k), static_cast<const __half *>(v), k_head_stride,
                            v_head_stride, static_cast<__half *>(output), (cudaStream_t)stream));
}

// ------------------------------------------------------------------------------------------
// Fused single-token attention half (Attention::forward, src/model.rs:79-162, T = 1).
// ------------------------------------------------------------------------------------------
namespace {
struct AttnLayout {
    size_t proj, part, out, vy, xq, tickets, total;
};
AttnLayout attn_layout(const MmrsAttnWeights *w) {
    const size_t qr = (size_t)w->query_heads * kAttnHeadDim, kr = (size_t)w->kv_heads * kAttnHeadDim;
    AttnLayout l{};
    size_t o = 0;
    auto take = [&](size_t b) {
        const size_t at = o;
        o = (o + b + 255) / 256 * 256;
        return at;
    };
    l.tickets = take(sizeof(uint32_t) * (2 + (size_t)w->kv_heads));  // [0] status, [1] pad, then one per KV head
    l.proj = take(sizeof(float) * (qr + 2 * kr));
    l.part = take(sizeof(float) * kAttnMaxSplits * w->query_heads * kAttnPartial);
    l.out = take(sizeof(__half) * qr);
    l.vy = take((qr / 32) * 36);
    l.xq = take(((size_t)w->hidden / 32) * 36);
    l.total = o;
    return l;
}
int attn_validate(const MmrsAttnWeights *w) {
    if (!w || !w->wq || !w->wk || !w->wv || !w->wo || !w->q_norm || !w->k_norm || !w->rope_cos || !w->rope_sin)
        return MMRS_ERR_ARG;
    if (w->hidden <= 0 || w->hidden % 64 || w->hidden > kMvMaxK || w->kv_heads < 1 ||
        w->query_heads != kAttnGroup * w->kv_heads || w->query_heads * kAttnHeadDim > kMvMaxK || w->rope_dim < 0 ||
        w->rope_dim > kAttnHeadDim || w->rope_dim % 2 || w->max_positions < 1)
        return MMRS_ERR_UNSUPPORTED;
    return MMRS_OK;
}
}  // namespace

extern "C" size_t mmrs_attn_workspace_bytes(const MmrsAttnWeights *w) {
    return attn_validate(w) == MMRS_OK ? attn_layout(w).total : 0;
}

extern "C" int mmrs_attn_workspace_status(const void *workspace) {
    if (!workspace) return MMRS_ERR_ARG;
    uint32_t st = 0;
    if (cudaMemcpy(&st, workspace, sizeof(st), cudaMemcpyDeviceToHost) != cudaSuccess) return MMRS_ERR_LAUNCH;
    return (int)st;
}

// Four launches, the last three allowed to start while their predecessor drains (programmatic
// dependent launch): the activation to Q8_1; the Q / K / V matvec (its weights streamed into
// shared memory before the wait); the GQA kernel in fused mode (cached K / V tiles requested
// before the wait; norm, RoPE, append, split merge and the Q8_1 output inside); the output
// projection on those Q8_1 blocks (+ residual).
extern "C" int mmrs_attn_decode_forward(const MmrsAttnWeights *w, const float *x, const float *residual, int position,
                                        void *k_cache, void *v_cache, float *y, void *workspace,
                                        size_t workspace_bytes, mmrs_stream_t stream) {
    int rc = attn_validate(w);
    if (rc != MMRS_OK) return rc;
    if (!x || !k_cache || !v_cache || !y || !workspace || position < 0 || position >= w->max_positions)
        return MMRS_ERR_ARG;
    const AttnLayout l = attn_layout(w);
    if (workspace_bytes < l.total || ((uintptr_t)workspace & 255u) || ((uintptr_t)k_cache & 15u) ||
        ((uintptr_t)v_cache & 15u))
        return MMRS_ERR_ARG;
    cudaStream_t s = (cudaStream_t)stream;
    uint8_t *ws = static_cast<uint8_t *>(workspace);
    float *proj = reinterpret_cast<float *>(ws + l.proj);
    const int qr = w->query_heads * kAttnHeadDim, kr = w->kv_heads * kAttnHeadDim;
    const long head_stride = (long)w->max_positions * kAttnHeadDim;
    // 1. Q / K / V projection (one launch for the three matrices)
    uint32_t *status = reinterpret_cast<uint32_t *>(ws + l.tickets);
    rc = qkv_launch(x, ws + l.xq, w->wq, w->wk, w->wv, proj, w->hidden, w->hidden, qr, kr, kr, s, status);
    if (rc != MMRS_OK) return rc;
    // 2. attention over positions [0, position]: about one CTA per SM, at least 4 chunks per split
    const int seq = position + 1, nch = (seq + kGqKeys - 1) / kGqKeys;
    const int splits = std::max(1, std::min({sm_count() / w->kv_heads, (nch + 7) / 8, kGqMaxFusedSplits}));
    CUtensorMap kmap, vmap;
    rc = make_kv_map(&kmap, k_cache, seq, w->kv_heads, head_stride);
    if (rc == MMRS_OK) rc = make_kv_map(&vmap, v_cache, seq, w->kv_heads, head_stride);
    if (rc != MMRS_OK) return rc;
    GqaParams g = {};
    g.proj = proj;
    g.q_norm = w->q_norm;
    g.k_norm = w->k_norm;
    g.cos = w->rope_cos;
    g.sin = w->rope_sin;
    g.eps = w->eps;
    g.rope_dim = w->rope_dim;
    g.k_cache = static_cast<__half *>(k_cache);
    g.v_cache = static_cast<__half *>(v_cache);
    g.cache_head_stride = head_stride;
    g.status = status;
    g.tickets = status + 2;
    g.out = reinterpret_cast<__half *>(ws + l.out);
    g.vy = ws + l.vy;
    g.partials = reinterpret_cast<float *>(ws + l.part);
    g.seq_len = seq;
    g.num_splits = splits;
    g.query_heads = w->query_heads;
    g.scale = 1.0f / sqrtf((float)kAttnHeadDim);
    gqa_smem_setup();
    if (launch_pdl(gqa_tc_kernel<true>, dim3(splits, w->kv_heads), dim3(kGqThreads), kGqSmemBytes, s, kmap, vmap, g) !=
        cudaSuccess)
        return MMRS_ERR_LAUNCH;
    // 3. output projection of the attention output's Q8_1 blocks (+ residual)
    MvParams o = {};
    o.w[0] = static_cast<const uint8_t *>(w->wo);
    o.n[0] = w->hidden;
    o.k = qr;
    o.kpad = qr;
    o.vy_in = ws + l.vy;
    o.residual = residual;
    o.dst = y;
    o.status = status;
    o.pre = kMsSlots;  // Wo does not depend on the attention kernel: stream it while that runs
    return mv_launch<float>(o, s);
}
