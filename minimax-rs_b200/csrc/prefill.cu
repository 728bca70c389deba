// Multi-token MoE path on B200: router GEMM for T tokens, sigmoid top-8, stable route bucketing,
// gathered Q8_1 quantisation (both reference numerics) and the grouped expert GEMM on tcgen05.
//
// Reference path (minimax-rs): FusedMoeGGUF::forward for T > 1 (fused_moe.rs:251-334):
// routing_flattened (fused_moe.rs:228-241), sort_routes (moe.rs:28-80, moe_sort.cu:21-51),
// moe_gemm_gguf for T < 32 (moe_gguf.cu:127-196, 357-424) and moe_gemm_mmq_gguf for T >= 32
// (mmq_moe.cu:69-165), SiLU * up, the weighted top-8 sum and the residual add (model.rs:218).
#include <cudaTypedefs.h>

#include <mutex>

#include "prefill.cuh"
#include "tma.cuh"
#include "umma.cuh"

namespace mmrs {

// ==========================================================================================
// 1. Router logits for T tokens in the canonical order shared with the decode kernel and the
//    CPU oracle: K is cut into 8 slices; in slice s lane l accumulates the float4 groups l,
//    l+32, l+64 of the slice with fmaf; the 32 lane partials are combined by an xor butterfly
//    (16, 8, 4, 2, 1) and the slices by ((s0+s1)+(s2+s3))+((s4+s5)+(s6+s7)).
//    Block: 8 warps = 8 slices, 8 experts per warp (weights in registers), 32 tokens per block.
//    Each warp streams its slice of the token rows through a kRtDepth-deep cp.async ring in
//    shared memory (a lane reads back exactly the 16-byte groups it copied), so the L2 latency
//    of token t+kRtDepth overlaps the arithmetic of token t.
//    The 8 butterflies of a warp are folded into one transposed reduction that produces the
//    same sums (each step adds the same two operands as the plain butterfly).
// ==========================================================================================
constexpr int kRtExperts = 8, kRtTokens = 32, kRtMaxIter = 3, kRtDepth = 3;  // H <= 3072

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

template <int ITER>
__global__ void __launch_bounds__(256) router_logits_kernel(const float *__restrict__ x,
                                                            const float *__restrict__ wr, int T, int E, int H,
                                                            float *__restrict__ logits) {
    __shared__ float part[kRtTokens][kRtExperts][8];
    __shared__ __align__(16) float4 ring[8][kRtDepth][32 * ITER];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int e0 = blockIdx.x * kRtExperts, t0 = blockIdx.y * kRtTokens;
    const int slice = H / 8, groups = slice / 4;
    const int tn = min(kRtTokens, T - t0);
    // token rows are only read through the ring; start the first kRtDepth copies before the
    // weight loads so both latencies overlap
    auto issue = [&](int tt) {
        if (tt < tn) {
            const float4 *src = reinterpret_cast<const float4 *>(x + (size_t)(t0 + tt) * H + warp * slice);
#pragma unroll
            for (int it = 0; it < ITER; ++it) {
                const int g = lane + 32 * it;
                if (g < groups) cp_async16(&ring[warp][tt % kRtDepth][g], src + g);
            }
        }
        cp_async_commit();  // one group per token slot, empty past the end
    };
#pragma unroll
    for (int d = 0; d < kRtDepth; ++d) issue(d);
    float4 w[kRtExperts][ITER];
#pragma unroll
    for (int e = 0; e < kRtExperts; ++e)
#pragma unroll
        for (int it = 0; it < ITER; ++it) {
            const int g = lane + 32 * it;
            w[e][it] = (g < groups && e0 + e < E)
                           ? __ldg(reinterpret_cast<const float4 *>(wr + (size_t)(e0 + e) * H + warp * slice) + g)
                           : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    for (int tt = 0; tt < tn; ++tt) {
        cp_async_wait<kRtDepth - 1>();  // this lane's copies of token tt have landed
        float4 xv[ITER];
#pragma unroll
        for (int it = 0; it < ITER; ++it) {
            const int g = lane + 32 * it;
            xv[it] = g < groups ? ring[warp][tt % kRtDepth][g] : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        float v[kRtExperts];
#pragma unroll
        for (int e = 0; e < kRtExperts; ++e) {
            float acc = 0.0f;
#pragma unroll
            for (int it = 0; it < ITER; ++it) {
                if (lane + 32 * it < groups) {
                    acc = fmaf(w[e][it].x, xv[it].x, acc);
                    acc = fmaf(w[e][it].y, xv[it].y, acc);
                    acc = fmaf(w[e][it].z, xv[it].z, acc);
                    acc = fmaf(w[e][it].w, xv[it].w, acc);
                }
            }
            v[e] = acc;
        }
        // transposed butterfly: after the xor-16 step a lane keeps 4 experts, after xor-8 two,
        // after xor-4 one; every kept value equals the plain butterfly's value at that lane.
        const int b4 = (lane >> 4) & 1, b3 = (lane >> 3) & 1, b2 = (lane >> 2) & 1;
        float a[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float send = b4 ? v[i] : v[4 + i];
            const float mine = b4 ? v[4 + i] : v[i];
            a[i] = mine + __shfl_xor_sync(0xffffffffu, send, 16);
        }
        float c[2];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const float send = b3 ? a[i] : a[2 + i];
            const float mine = b3 ? a[2 + i] : a[i];
            c[i] = mine + __shfl_xor_sync(0xffffffffu, send, 8);
        }
        float d;
        {
            const float send = b2 ? c[0] : c[1];
            const float mine = b2 ? c[1] : c[0];
            d = mine + __shfl_xor_sync(0xffffffffu, send, 4);
        }
        d = d + __shfl_xor_sync(0xffffffffu, d, 2);
        d = d + __shfl_xor_sync(0xffffffffu, d, 1);
        if ((lane & 3) == 0) part[tt][4 * b4 + 2 * b3 + b2][warp] = d;
        issue(tt + kRtDepth);  // the slot's values are consumed (d depends on them)
    }
    cp_async_wait<0>();
    __syncthreads();
    for (int i = threadIdx.x; i < tn * kRtExperts; i += blockDim.x) {
        const int tt = i / kRtExperts, e = i % kRtExperts;
        if (e0 + e >= E) continue;
        const float *s = part[tt][e];
        logits[(size_t)(t0 + tt) * E + e0 + e] = ((s[0] + s[1]) + (s[2] + s[3])) + ((s[4] + s[5]) + (s[6] + s[7]));
    }
}

int pf_router_logits(const float *x, const float *router, int T, int E, int H, float *logits, cudaStream_t s) {
    if (T <= 0) return MMRS_OK;
    if (H % QK_K || H > 1024 * kRtMaxIter) return MMRS_ERR_UNSUPPORTED;
    const dim3 grid((E + kRtExperts - 1) / kRtExperts, (T + kRtTokens - 1) / kRtTokens);
    const int iter = (H / 32 + 31) / 32;
    if (iter == 1)
        router_logits_kernel<1><<<grid, 256, 0, s>>>(x, router, T, E, H, logits);
    else if (iter == 2)
        router_logits_kernel<2><<<grid, 256, 0, s>>>(x, router, T, E, H, logits);
    else
        router_logits_kernel<3><<<grid, 256, 0, s>>>(x, router, T, E, H, logits);
    return cudaGetLastError() == cudaSuccess ? MMRS_OK : MMRS_ERR_LAUNCH;
}

// ==========================================================================================
// 2. Sigmoid top-8 per token (routing_flattened, fused_moe.rs:228-241): s = 1/(1+expf(-l)),
//    selection by s + bias in stable descending order (lower expert id first on ties),
//    weights s / tree-sum (strides 4, 2, 1).  One warp per token.
// ==========================================================================================
template <int kPer>  // experts per lane: E <= 32 * kPer
__global__ void __launch_bounds__(256) route_topk_kernel(const float *__restrict__ logits,
                                                         const float *__restrict__ bias, int T, int E,
                                                         uint32_t *__restrict__ ids, float *__restrict__ wts) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * 8 + warp;
    if (t >= T) return;
    float sel[kPer], sig[kPer];
    const int per = (E + 31) / 32;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
        const int e = lane + 32 * i;
        if (i < per && e < E) {
            const float sg = __fdiv_rn(1.0f, 1.0f + expf(-logits[(size_t)t * E + e]));
            float sv = sg + bias[e];
            if (sv == 0.0f) sv = 0.0f;  // -0 ranks as +0
            sig[i] = sg;
            sel[i] = sv;
        } else {
            sig[i] = 0.0f;
            sel[i] = -INFINITY;
        }
    }
    uint32_t taken = 0;  // bit i: expert lane + 32 i already selected
    float picked[8];
    int pid[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        float best = -INFINITY;
        int bi = -1;
#pragma unroll
        for (int i = 0; i < kPer; ++i) {
            const int e = lane + 32 * i;
            if (i < per && e < E && !((taken >> i) & 1u) && (bi < 0 || sel[i] > best)) {
                best = sel[i];
                bi = i;
            }
        }
        int be = bi < 0 ? 0x7fffffff : lane + 32 * bi;
        // warp arg-max: larger value wins, equal values -> lower expert id
#pragma unroll
        for (int m = 16; m > 0; m >>= 1) {
            const float ob = __shfl_xor_sync(0xffffffffu, best, m);
            const int oe = __shfl_xor_sync(0xffffffffu, be, m);
            if (oe != 0x7fffffff && (be == 0x7fffffff || ob > best || (ob == best && oe < be))) {
                best = ob;
                be = oe;
            }
        }
        pid[k] = be;
        float sgv = 0.0f;
        if ((be & 31) == lane) {
            const int i = be >> 5;
#pragma unroll
            for (int q = 0; q < kPer; ++q)
                if (q == i) {
                    sgv = sig[q];
                    taken |= 1u << q;
                }
        }
        picked[k] = __shfl_sync(0xffffffffu, sgv, be & 31);
    }
    if (lane == 0) {
        const float denom = ((picked[0] + picked[4]) + (picked[2] + picked[6])) +
                            ((picked[1] + picked[5]) + (picked[3] + picked[7]));
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            ids[(size_t)t * 8 + k] = (uint32_t)pid[k];
            wts[(size_t)t * 8 + k] = __fdiv_rn(picked[k], denom);
        }
    }
}

int pf_route_topk(const float *logits, const float *bias, int T, int E, uint32_t *ids, float *w, cudaStream_t s) {
    if (T <= 0) return MMRS_OK;
    if (E < 8 || E > kPfMaxExperts) return MMRS_ERR_UNSUPPORTED;
    const unsigned blocks = (T + 7) / 8;
    if (E <= 256)
        route_topk_kernel<8><<<blocks, 256, 0, s>>>(logits, bias, T, E, ids, w);
    else
        route_topk_kernel<kPfMaxExperts / 32><<<blocks, 256, 0, s>>>(logits, bias, T, E, ids, w);
    return cudaGetLastError() == cudaSuccess ? MMRS_OK : MMRS_ERR_LAUNCH;
}

// ==========================================================================================
// 3. Stable sort of route keys (moe_sort_routes: CUB radix sort of (key, route) pairs on bits
//    [0, end_bit), moe_sort.cu:21-51).  One CTA: histogram, exclusive scan, then rounds of
//    1024 keys in index order; inside a round a key's position is its bucket base + the count
//    of equal buckets in lower warps + its rank among equal buckets of its own warp.
// ==========================================================================================
constexpr int kSortMaxBits = 10;

__global__ void __launch_bounds__(1024) sort_routes_kernel(const uint32_t *__restrict__ keys, int n, int end_bit,
                                                           uint32_t *__restrict__ sorted_keys,
                                                           uint32_t *__restrict__ sorted_routes) {
    extern __shared__ uint8_t sm_sort[];
    const int nb = 1 << end_bit;
    const uint32_t mask = (uint32_t)nb - 1u;
    int *base = reinterpret_cast<int *>(sm_sort);
    uint16_t *wcnt = reinterpret_cast<uint16_t *>(base + nb);  // [32][nb]
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    for (int b = tid; b < nb; b += blockDim.x) base[b] = 0;
    for (int i = tid; i < 32 * nb; i += blockDim.x) wcnt[i] = 0;
    __syncthreads();
    for (int i = tid; i < n; i += blockDim.x) atomicAdd(&base[keys[i] & mask], 1);
    __syncthreads();
    if (tid == 0) {  // exclusive scan (nb <= 1024)
        int run = 0;
        for (int b = 0; b < nb; ++b) {
            const int c = base[b];
            base[b] = run;
            run += c;
        }
    }
    __syncthreads();
    const uint32_t lt = (1u << lane) - 1u;
    for (int r0 = 0; r0 < n; r0 += blockDim.x) {
        const int i = r0 + tid;
        const bool act = i < n;
        const uint32_t key = act ? keys[i] : 0u;
        const int b = act ? (int)(key & mask) : -1;
        const uint32_t peers = __match_any_sync(0xffffffffu, b);
        const int rank = __popc(peers & lt);
        const bool leader = act && rank == 0;
        if (leader) wcnt[warp * nb + b] = (uint16_t)__popc(peers);
        __syncthreads();
        if (act) {
            int off = base[b] + rank;
            for (int w = 0; w < warp; ++w) off += wcnt[w * nb + b];
            sorted_keys[off] = key;
            sorted_routes[off] = (uint32_t)i;
        }
        __syncthreads();
        if (leader) {
            atomicAdd(&base[b], __popc(peers));
            wcnt[warp * nb + b] = 0;
        }
        __syncthreads();
    }
}

int pf_sort_routes(const uint32_t *keys, int n, int end_bit, uint32_t *sorted_keys, uint32_t *sorted_routes,
                   cudaStream_t s) {
    if (n <= 0) return MMRS_OK;
    if (end_bit < 0) return MMRS_ERR_ARG;
    if (end_bit > kSortMaxBits) return MMRS_ERR_UNSUPPORTED;
    const size_t smem = sizeof(int) * (1 << end_bit) + sizeof(uint16_t) * 32 * (1 << end_bit);
    static std::once_flag once[64];
    int dev = 0;
    cudaGetDevice(&dev);
    std::call_once(once[dev & 63], [] {
        cudaFuncSetAttribute(sort_routes_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)(sizeof(int) * 1024 + sizeof(uint16_t) * 32 * 1024));
    });
    sort_routes_kernel<<<1, 1024, smem, s>>>(keys, n, end_bit, sorted_keys, sorted_routes);
    return cudaGetLastError() == cudaSuccess ? MMRS_OK : MMRS_ERR_LAUNCH;
}

// ==========================================================================================
// 4. Bucketing plan from an expert-sorted route list (the contract of the reference's
//    sorted_token_ids / expert_ids arguments): per-expert count and first position by binary
//    search, 16-row padded segments, tile prefix, and the padded row -> route map.
// ==========================================================================================
__device__ __forceinline__ int lower_bound_i32(const int32_t *a, int n, int v) {
    int lo = 0, hi = n;
    while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (a[mid] < v) lo = mid + 1;
        else hi = mid;
    }
    return lo;
}

__device__ __forceinline__ int block_excl_scan_1024(int v, int *tmp /* >= 32 ints */, int &total) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int inc = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += y;
    }
    if (lane == 31) tmp[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        const int wv = lane < (int)(blockDim.x >> 5) ? tmp[lane] : 0;
        int wi = wv;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, wi, o);
            if (lane >= o) wi += y;
        }
        tmp[lane] = wi - wv;  // exclusive prefix of warp totals
        if (lane == 31) tmp[32] = wi;
    }
    __syncthreads();
    const int r = tmp[warp] + inc - v;
    total = tmp[32];
    __syncthreads();
    return r;
}

__global__ void __launch_bounds__(1024) build_plan_kernel(const int32_t *__restrict__ se,
                                                          const int32_t *__restrict__ sr, int M, int E,
                                                          PfPlan plan, int own_world, int own_rank) {
    __shared__ int tmp[33];
    __shared__ int s_first[kPfMaxExperts], s_seg[kPfMaxExperts];
    const int e = threadIdx.x;
    int first = 0, cnt = 0;
    if (e < E) {
        first = lower_bound_i32(se, M, e);
        cnt = e % own_world == own_rank ? lower_bound_i32(se, M, e + 1) - first : 0;
    }
    int total;
    const int seg = block_excl_scan_1024(e < E ? pad_to(cnt, kPfSegAlign) : 0, tmp, total);
    const int tl = block_excl_scan_1024(e < E ? (cnt + kPfNT - 1) / kPfNT : 0, tmp, total);
    if (e < E) {
        plan.count[e] = cnt;
        plan.first[e] = first;
        plan.seg[e] = seg;
        plan.tiles[e] = tl;
        s_first[e] = first;
        s_seg[e] = seg;
    }
    if (e == 0) plan.tiles[E] = total;
    for (int p = threadIdx.x; p < plan.ppad; p += blockDim.x) plan.row_route[p] = -1;
    __syncthreads();
    for (int i = threadIdx.x; i < M; i += blockDim.x) {
        const int ex = se[i];
        if (ex < 0 || ex >= E || ex % own_world != own_rank) continue;
        plan.row_route[s_seg[ex] + i - s_first[ex]] = sr[i];
    }
}

int pf_build_plan(const int32_t *sorted_experts, const int32_t *sorted_routes, int M, int E, PfPlan plan,
                  cudaStream_t s, int own_world, int own_rank) {
    if (E < 1 || E > kPfMaxExperts) return MMRS_ERR_UNSUPPORTED;
    if (own_world < 1 || own_rank < 0 || own_rank >= own_world) return MMRS_ERR_ARG;
    build_plan_kernel<<<1, 1024, 0, s>>>(sorted_experts, sorted_routes, M, E, plan, own_world, own_rank);
    return cudaGetLastError() == cudaSuccess ? MMRS_OK : MMRS_ERR_LAUNCH;
}

// ==========================================================================================
// 5. Gathered Q8_1 quantisation into the operand layout (one warp per padded row and 256-column
//    chunk; lane = 4 consecutive values, 8 lanes = one 32-block).
//    MMQ (quantize_mmq_q8_1<DS4>, mmq_quantize.cu:59-72): d_inv = 127/amax, q = roundf(x*d_inv),
//      d = half(1/d_inv), s = half(((x0+x1)+x2)+x3 then xor 4, 2, 1 over the 8 lanes).
//    Generic (quantize_q8_1, gguf.cuh:1234-1261): d = amax/127, q = roundf(x/d);
//      the dot combine uses d8 = half(d) and s8 = d8 * sum(q) (vec_dot_q4_K_q8_1_impl_vmmq).
// ==========================================================================================
__global__ void __launch_bounds__(256) quantize_rows_kernel(const float *__restrict__ x,
                                                            const float *__restrict__ x2, int div, int K,
                                                            int mode, PfPlan plan, PfActs acts) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const int nkc = K / QK_K;
    const int p = warp / nkc, kc = warp % nkc;
    if (p >= plan.ppad) return;
    const int route = plan.row_route[p];
    if (route < 0) return;
    const int src = x2 ? route : route / div;
    const int grp = lane >> 3;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
        const int kk = half * 128 + lane * 4;  // column inside the chunk
        const size_t gi = (size_t)src * K + (size_t)kc * QK_K + kk;
        float4 v = *reinterpret_cast<const float4 *>(x + gi);
        if (x2) {
            const float4 u = *reinterpret_cast<const float4 *>(x2 + gi);
            v.x = __fmul_rn(u.x, __fdiv_rn(v.x, 1.0f + expf(-v.x)));
            v.y = __fmul_rn(u.y, __fdiv_rn(v.y, 1.0f + expf(-v.y)));
            v.z = __fmul_rn(u.z, __fdiv_rn(v.z, 1.0f + expf(-v.z)));
            v.w = __fmul_rn(u.w, __fdiv_rn(v.w, 1.0f + expf(-v.w)));
        }
        float amax = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
#pragma unroll
        for (int m = 4; m > 0; m >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, m));
        int q0, q1, q2, q3;
        float d8, s8;
        if (mode == kPfModeMmq) {
            float t = ((v.x + v.y) + v.z) + v.w;
#pragma unroll
            for (int m = 4; m > 0; m >>= 1) t = t + __shfl_xor_sync(0xffffffffu, t, m);
            if (amax == 0.0f) {
                q0 = q1 = q2 = q3 = 0;
                d8 = 0.0f;
            } else {
                const float dinv = __fdiv_rn(127.0f, amax);
                q0 = (int)roundf(__fmul_rn(v.x, dinv));
                q1 = (int)roundf(__fmul_rn(v.y, dinv));
                q2 = (int)roundf(__fmul_rn(v.z, dinv));
                q3 = (int)roundf(__fmul_rn(v.w, dinv));
                d8 = __half2float(__float2half_rn(__fdiv_rn(1.0f, dinv)));
            }
            s8 = __half2float(__float2half_rn(t));
        } else {
            const float d = __fdiv_rn(amax, 127.0f);
            if (amax == 0.0f) {
                q0 = q1 = q2 = q3 = 0;
            } else {
                q0 = (int)roundf(__fdiv_rn(v.x, d));
                q1 = (int)roundf(__fdiv_rn(v.y, d));
                q2 = (int)roundf(__fdiv_rn(v.z, d));
                q3 = (int)roundf(__fdiv_rn(v.w, d));
            }
            int qs = q0 + q1 + q2 + q3;
#pragma unroll
            for (int m = 4; m > 0; m >>= 1) qs += __shfl_xor_sync(0xffffffffu, qs, m);
            d8 = __half2float(__float2half_rn(d));
            s8 = __fmul_rn(d8, (float)qs);
        }
        const uint32_t word = (uint32_t)(q0 & 0xff) | ((uint32_t)(q1 & 0xff) << 8) | ((uint32_t)(q2 & 0xff) << 16) |
                              ((uint32_t)(q3 & 0xff) << 24);
        const size_t off = (size_t)kc * plan.ppad * QK_K + (size_t)(p >> 3) * 2048 + (kk >> 4) * 128 + (p & 7) * 16 +
                           (kk & 15);
        *reinterpret_cast<uint32_t *>(acts.q + off) = word;
        if ((lane & 7) == 0) {
            float *rec = acts.ds + ((size_t)kc * (plan.ppad / 16) + p / 16) * 256 + (half * 4 + grp) * 16 + p % 16;
            rec[0] = d8;
            rec[128] = s8;
        }
    }
}

int pf_quantize(const float *x, const float *x2, int div, int K, int mode, PfPlan plan, PfActs acts, int rows_max,
                cudaStream_t s) {
    if (rows_max <= 0) return MMRS_OK;
    if (K % QK_K) return MMRS_ERR_ARG;
    const long warps = (long)rows_max * (K / QK_K);
    const long blocks = (warps * 32 + 255) / 256;
    quantize_rows_kernel<<<(unsigned)blocks, 256, 0, s>>>(x, x2, div, K, mode, plan, acts);
    return cudaGetLastError() == cudaSuccess ? MMRS_OK : MMRS_ERR_LAUNCH;
}

// ==========================================================================================
// 6. Weighted top-k sum + residual: y[t] = (sum_k dn[t*8+k], k ascending) + residual[t]
//    (the `sum(-2)` of fused_moe.rs:327-328 and the residual add of model.rs:218).
// ==========================================================================================
__global__ void __launch_bounds__(256) reduce_topk_kernel(const float *__restrict__ dn,
                                                          const float *__restrict__ residual, int T, int H,
                                                          float *__restrict__ y, const uint32_t *__restrict__ ids,
                                                          int own_world, int own_rank) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;  // float4 index
    const size_t n4 = (size_t)T * H / 4;
    if (i >= n4) return;
    const size_t t = (i * 4) / H, h = (i * 4) % H;
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        if (own_world > 1 && ids[t * 8 + k] % (uint32_t)own_world != (uint32_t)own_rank) continue;
        const float4 v = *reinterpret_cast<const float4 *>(dn + ((t * 8 + k) * H + h));
        s.x = s.x + v.x;
        s.y = s.y + v.y;
        s.z = s.z + v.z;
        s.w = s.w + v.w;
    }
    if (residual) {
        const float4 r = *reinterpret_cast<const float4 *>(residual + t * H + h);
        s.x = s.x + r.x;
        s.y = s.y + r.y;
        s.z = s.z + r.z;
        s.w = s.w + r.w;
    }
    *reinterpret_cast<float4 *>(y + t * H + h) = s;
}

int pf_reduce_topk(const float *dn, const float *residual, int T, int H, float *y, cudaStream_t s,
                   const uint32_t *ids, int own_world, int own_rank) {
    if (T <= 0) return MMRS_OK;
    if (own_world > 1 && !ids) return MMRS_ERR_ARG;
    const size_t n4 = (size_t)T * H / 4;
    reduce_topk_kernel<<<(unsigned)((n4 + 255) / 256), 256, 0, s>>>(dn, residual, T, H, y, ids, own_world, own_rank);
    return cudaGetLastError() == cudaSuccess ? MMRS_OK : MMRS_ERR_LAUNCH;
}

// ==========================================================================================
// 7. Grouped expert GEMM on tcgen05 (kind::i8, accumulators in TMEM).
//
//    Work item = (expert e, route tile of <= 32 routes, 128 weight rows).  Per 256-column chunk
//    (one GGUF super-block of every row):
//      warp 0      TMA: the raw weight tile (tensor map, 128 rows x one super-block) and the route
//                  tile's block scales into the raw ring; the route tile's int8 activations
//                  (B operand) into the operand stage
//      warps 2-5   unpack (one thread per row): nibbles (+ high bits) -> int8 A operand in the
//                  canonical no-swizzle K-major shared-memory layout; per 32-block and row the
//                  scales (dmx, dmy); the route tile's (d8, s8) planes for the epilogue
//      warp 1      one thread issues the chunk's 8 MMAs (M=128, N=routes rounded to 16, K=32),
//                  one per 32-block, each into its own accumulator of the chunk's TMEM group
//                  (8 x 32 columns), then one commit for the group
//      warps 6-21  epilogue: 4 TMEM lane quarters x 4 units of 8 route columns; per 32-block
//                  sum = fma(dmx * d8, C, sum); sum = fma(dmy, s8, sum) in K order (the MMQ combine
//                  of mmq_gguf.cuh vec_dot_q8_1_q8_1_mma, or with the generic numerics' scales the
//                  vec_dot_q*_K_q8_1 combine), then the route rows are written (times the route
//                  weight when given).
//    Integer accumulators without a conversion: every accumulator column holds the bit pattern
//    of 1.5 * 2^23 (0x4B400000) before its MMA, which adds the block's integer dot product C
//    (|C| <= 32 * 31 * 127 < 2^22) to it, so the column reads as the float 12582912 + C and one
//    exact subtraction gives C.  The epilogue writes the pattern back after reading a column.
//    Every wait is bounded by a %globaltimer deadline; on expiry the CTA records
//    MMRS_ERR_TIMEOUT, stops, waits (bounded) for its own copies and MMAs and frees its TMEM.
// ==========================================================================================
constexpr int kPfRawW = kPfMT * Q5K_BYTES;      // 22528: raw weight tile
constexpr int kPfRawQ = kPfNT * QK_K;           // 8192: int8 activations of the route tile (B operand)
constexpr int kPfRawD = kPfNT * 8 * 8;          // 2048: d8 and s8 planes of the route tile
constexpr int kPfRawBytes = kPfRawW + kPfRawD;
constexpr int kPfABytes = kPfMT * QK_K;         // 32768
constexpr int kPfEpiWarp0 = 2 + kPfUnpackWarps;
constexpr int kPfGroupCols = 8 * kPfNT;         // 256: the 8 block accumulators of one chunk
constexpr int kPfTmemCols = kPfGroups * kPfGroupCols;
static_assert(kPfTmemCols == 512, "two chunk groups fill the tensor memory");
static_assert(kPfNT == 32 && kPfEpiWarps == 16, "epilogue geometry: 4 lane quarters x 4 x 8 route columns");
constexpr int kPfPrefetch = 6;                  // weight tiles prefetched to L2 ahead of the loads
constexpr uint32_t kPfAccBias = 0x4B400000u;  // float 12582912 = 1.5 * 2^23
constexpr float kPfAccBiasF = 12582912.0f;

// Raw stage (TMA / bulk copies): the weights and the activation block scales of one chunk; it is
// free again as soon as the unpack warps have read it.
// Operand stage: the MMA operands (A from the unpack warps, B by a bulk copy; free when the
// chunk's MMAs complete) and the epilogue's scales (free when the epilogue has used them).
struct PfSmem {
    uint8_t raw[kPfRawStages][kPfRawBytes];
    uint8_t a[kPfOpStages][kPfABytes];
    uint8_t b[kPfOpStages][kPfRawQ];
    float2 sc[kPfOpStages][8 * kPfMT];       // (dmx, dmy) per 32-block and row
    float dst[kPfOpStages][2][8][kPfNT];     // [d8 | s8][32-block][route]
    uint64_t rfull[kPfRawStages], rempty[kPfRawStages];
    uint64_t bfull[kPfOpStages], abempty[kPfOpStages], sdempty[kPfOpStages], aready[kPfOpStages];
    uint64_t gfull[kPfGroups], gfree[kPfGroups];
    uint64_t mdone;
    int tiles[kPfMaxExperts + 1];            // route-tile prefix of the plan (item decoding)
    uint32_t tmem_base;
    int abort;
};

static_assert(sizeof(PfSmem) + 128 <= 232448, "PfSmem exceeds the 227 KB a CTA can opt in to");
size_t pf_gemm_smem_bytes() { return sizeof(PfSmem) + 128; }

__device__ __forceinline__ void tc_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tc_ld8(uint32_t taddr, uint32_t (&v)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(taddr));
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_st8_const(uint32_t taddr, uint32_t v) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(taddr), "r"(v)
                 : "memory");
}
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tma_prefetch_2d(const CUtensorMap *map, int x, int y) {
    asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(x), "r"(y)
                 : "memory");
}

struct PfItem {
    int e, p0, nvalid, m0;
};
__device__ __forceinline__ PfItem pf_item(const PfGemmParams &p, const int *tiles, int item) {
    PfItem it;
    const int et = item / p.mt;
    it.m0 = (item % p.mt) * kPfMT;
    int lo = 0, hi = p.E;  // largest e with tiles[e] <= et
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (tiles[mid] <= et) lo = mid;
        else hi = mid;
    }
    it.e = lo;
    const int nt = et - tiles[lo];
    it.p0 = p.plan.seg[lo] + nt * kPfNT;
    it.nvalid = min(kPfNT, p.plan.count[lo] - nt * kPfNT);
    return it;
}

// Unpack one raw GGUF super-block row into the int8 A tile (canonical no-swizzle K-major layout:
// 8-row groups 2048 B apart, 16-byte K slices 128 B apart, rows 16 B apart) and its 8 scale
// pairs.  Every 16-byte load of the row is issued before the first store, so the loads are in
// flight together instead of each waiting behind the previous store.
template <int GT, int MODE>
__device__ __forceinline__ void pf_unpack_row(const uint8_t *__restrict__ blk, uint8_t *__restrict__ a_tile,
                                              float2 *__restrict__ sc_col, int r) {
    constexpr int kQs = GT == MMRS_Q5K ? 48 : 16;
    const uint4 hdr = *reinterpret_cast<const uint4 *>(blk);
    uint4 qh0 = make_uint4(0, 0, 0, 0), qh1 = make_uint4(0, 0, 0, 0);
    if (GT == MMRS_Q5K) {
        qh0 = *reinterpret_cast<const uint4 *>(blk + 16);
        qh1 = *reinterpret_cast<const uint4 *>(blk + 32);
    }
    uint4 qv[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) qv[q] = *reinterpret_cast<const uint4 *>(blk + kQs + 16 * q);

    uint8_t *arow = a_tile + (r >> 3) * 2048 + (r & 7) * 16;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
        const int jp = q >> 1, hf = q & 1;
        const uint4 v = qv[q];
        uint4 lo, hi;
        lo.x = v.x & 0x0F0F0F0Fu;
        lo.y = v.y & 0x0F0F0F0Fu;
        lo.z = v.z & 0x0F0F0F0Fu;
        lo.w = v.w & 0x0F0F0F0Fu;
        hi.x = (v.x >> 4) & 0x0F0F0F0Fu;
        hi.y = (v.y >> 4) & 0x0F0F0F0Fu;
        hi.z = (v.z >> 4) & 0x0F0F0F0Fu;
        hi.w = (v.w >> 4) & 0x0F0F0F0Fu;
        if (GT == MMRS_Q5K) {
            const uint4 h = hf ? qh1 : qh0;
            const int sl = 2 * jp, sh = 2 * jp + 1;
            lo.x |= ((h.x >> sl) & 0x01010101u) << 4;
            lo.y |= ((h.y >> sl) & 0x01010101u) << 4;
            lo.z |= ((h.z >> sl) & 0x01010101u) << 4;
            lo.w |= ((h.w >> sl) & 0x01010101u) << 4;
            hi.x |= ((h.x >> sh) & 0x01010101u) << 4;
            hi.y |= ((h.y >> sh) & 0x01010101u) << 4;
            hi.z |= ((h.z >> sh) & 0x01010101u) << 4;
            hi.w |= ((h.w >> sh) & 0x01010101u) << 4;
        }
        *reinterpret_cast<uint4 *>(arow + (4 * jp + hf) * 128) = lo;
        *reinterpret_cast<uint4 *>(arow + (4 * jp + 2 + hf) * 128) = hi;
    }
    const float dall = half_bits_to_float(hdr.x), dmin = half_bits_to_float(hdr.x >> 16);
    const uint32_t w0 = hdr.y, w1 = hdr.z, w2 = hdr.w;  // the 12 packed scale bytes
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        // get_scale_min_k4 (quantized.cu:926-933) on bytes of w0..w2
        const auto byte = [&](int i) -> uint32_t {
            const uint32_t w = i < 4 ? w0 : (i < 8 ? w1 : w2);
            return (w >> (8 * (i & 3))) & 0xffu;
        };
        uint32_t sc, mn;
        if (j < 4) {
            sc = byte(j) & 63;
            mn = byte(j + 4) & 63;
        } else {
            sc = (byte(j + 4) & 0xF) | ((byte(j - 4) >> 6) << 4);
            mn = (byte(j + 4) >> 4) | ((byte(j) >> 6) << 4);
        }
        float dmx = __fmul_rn(dall, small_uint_to_float(sc)), dmy = __fmul_rn(-dmin, small_uint_to_float(mn));
        if (MODE == kPfModeMmq) {  // the MMQ tile loader rounds both products to half
            const float2 h = __half22float2(__floats2half2_rn(dmx, dmy));
            dmx = h.x;
            dmy = h.y;
        }
        sc_col[j * kPfMT] = make_float2(dmx, dmy);
    }
}

__device__ __forceinline__ bool pf_aborted(PfSmem &sm) { return *reinterpret_cast<volatile int *>(&sm.abort) != 0; }

__device__ __forceinline__ bool pf_wait(uint64_t *bar, uint32_t parity, uint64_t deadline, PfSmem &sm,
                                        uint32_t *status) {
    if (mbar_wait_sleep(bar, parity, deadline)) return true;
    atomicExch(status, MMRS_ERR_TIMEOUT);
    *reinterpret_cast<volatile int *>(&sm.abort) = 1;
    return false;
}

// Packed fp32 pairs (two IEEE operations per instruction, the same results as the scalar forms).
__device__ __forceinline__ unsigned long long f2_bits(float2 v) { return *reinterpret_cast<unsigned long long *>(&v); }
__device__ __forceinline__ float2 bits_f2(unsigned long long v) { return *reinterpret_cast<float2 *>(&v); }
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    unsigned long long r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(f2_bits(a)), "l"(f2_bits(b)), "l"(f2_bits(c)));
    return bits_f2(r);
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
    unsigned long long r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(f2_bits(a)), "l"(f2_bits(b)));
    return bits_f2(r);
}
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
    unsigned long long r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(f2_bits(a)), "l"(f2_bits(b)));
    return bits_f2(r);
}

// Scales of one 32-block for 8 route columns: (dmx, dmy) of the row, d8 and s8 of the routes.
struct PfScales8 {
    float2 row;
    float4 d[2], s[2];
};
__device__ __forceinline__ PfScales8 pf_scales8(float2 row, const float *dcol, const float *scol) {
    PfScales8 z;
    z.row = row;
    z.d[0] = *reinterpret_cast<const float4 *>(dcol);
    z.d[1] = *reinterpret_cast<const float4 *>(dcol + 4);
    z.s[0] = *reinterpret_cast<const float4 *>(scol);
    z.s[1] = *reinterpret_cast<const float4 *>(scol + 4);
    return z;
}

// Scale-and-accumulate 8 route columns of one 32-block: per column
// sum = fma(dmx * d8, C, sum); sum = fma(dmy, s8, sum).
__device__ __forceinline__ void pf_accumulate8(float2 (&acc)[4], const uint32_t (&v)[8], const PfScales8 &z) {
    const float2 dmx = make_float2(z.row.x, z.row.x), dmy = make_float2(z.row.y, z.row.y);
#pragma unroll
    for (int h4 = 0; h4 < 2; ++h4) {
        const float2 dp[2] = {make_float2(z.d[h4].x, z.d[h4].y), make_float2(z.d[h4].z, z.d[h4].w)};
        const float2 sp[2] = {make_float2(z.s[h4].x, z.s[h4].y), make_float2(z.s[h4].z, z.s[h4].w)};
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int i = 2 * h4 + u;
            // exact C from the biased accumulator (see the bias note above the kernel)
            const float2 cf = fadd2(make_float2(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1])),
                                    make_float2(-kPfAccBiasF, -kPfAccBiasF));
            acc[i] = ffma2(fmul2(dmx, dp[u]), cf, acc[i]);
            acc[i] = ffma2(dmy, sp[u], acc[i]);
        }
    }
}

template <int GT, int MODE>
__global__ void __launch_bounds__(kPfThreads, 1) pf_gemm_kernel(const __grid_constant__ CUtensorMap wmap,
                                                                const PfGemmParams p) {
    extern __shared__ uint8_t sm_raw[];
    PfSmem &sm = *reinterpret_cast<PfSmem *>((reinterpret_cast<uintptr_t>(sm_raw) + 127) & ~uintptr_t(127));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int bb = GT == MMRS_Q5K ? Q5K_BYTES : Q4K_BYTES;
    const int nkc = p.K / QK_K;
    const int total = p.plan.tiles[p.E] * p.mt;
    const uint64_t deadline = globaltimer_ns() + p.timeout_ns;

    if (tid == 0) {
        for (int i = 0; i < kPfRawStages; ++i) {
            mbar_init(&sm.rfull[i], 1);
            mbar_init(&sm.rempty[i], kPfUnpackWarps);
        }
        for (int i = 0; i < kPfOpStages; ++i) {
            mbar_init(&sm.bfull[i], 1);
            mbar_init(&sm.abempty[i], 1);              // MMA commit
            mbar_init(&sm.sdempty[i], kPfEpiWarps);
            mbar_init(&sm.aready[i], kPfUnpackWarps);
        }
        for (int i = 0; i < kPfGroups; ++i) {
            mbar_init(&sm.gfull[i], 1);
            mbar_init(&sm.gfree[i], kPfEpiWarps);
        }
        mbar_init(&sm.mdone, 1);
        sm.abort = 0;
        fence_mbar_init();
    }
    for (int i = tid; i <= p.E; i += blockDim.x) sm.tiles[i] = p.plan.tiles[i];
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&sm.tmem_base)),
                     "r"(kPfTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sm.tmem_base;
    if (warp >= kPfEpiWarp0) {
        // every accumulator column starts at the bias pattern (each epilogue warp: its lane
        // quarter and route unit, all 8 blocks of both groups)
        const int qd = warp & 3, u = (warp - kPfEpiWarp0) >> 2;
        const uint32_t tq = tmem + ((uint32_t)(qd * 32) << 16) + 8 * u;
#pragma unroll
        for (int gj = 0; gj < kPfGroups * 8; ++gj) tc_st8_const(tq + gj * kPfNT, kPfAccBias);
        tc_wait_st();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            uint32_t c = 0, raw_extra = 0;
            // L2 prefetch cursor kPfPrefetch chunks ahead of the loads: the strided weight tile
            // (128 rows of one super-block) has a long DRAM latency that the raw ring alone
            // cannot cover
            int pitem = blockIdx.x, pkc = 0, prow0 = -1;
            const auto prefetch_next = [&]() {
                if (pitem >= total) return;
                if (pkc == 0) {
                    const PfItem pi = pf_item(p, sm.tiles, pitem);
                    prow0 = pi.e * p.N + pi.m0;
                }
                tma_prefetch_2d(&wmap, pkc * (bb / 4), prow0);
                if (++pkc == nkc) {
                    pkc = 0;
                    pitem += gridDim.x;
                }
            };
            for (int i = 0; i < kPfPrefetch; ++i) prefetch_next();
            for (int item = blockIdx.x; item < total && !pf_aborted(sm); item += gridDim.x) {
                const PfItem it = pf_item(p, sm.tiles, item);
                const int row0 = it.e * p.N + it.m0;
                const int n16 = pad_to(it.nvalid, 16);
                const uint32_t qb = (uint32_t)n16 * QK_K, db = (uint32_t)n16 * 64;
                bool ok = true;
                for (int kc = 0; kc < nkc; ++kc, ++c) {
                    const int s = c % kPfRawStages, o = c % kPfOpStages;
                    if (!pf_wait(&sm.rempty[s], ((c / kPfRawStages) & 1) ^ 1, deadline, sm, p.status)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&sm.rfull[s], (uint32_t)(kPfMT * bb) + db);
                    tma_load_2d(sm.raw[s], &wmap, kc * (bb / 4), row0, &sm.rfull[s]);
                    prefetch_next();
                    bulk_g2s(sm.raw[s] + kPfRawW, p.ads + ((size_t)kc * (p.plan.ppad / 16) + it.p0 / 16) * 256, db,
                             &sm.rfull[s]);
                    if (!pf_wait(&sm.abempty[o], ((c / kPfOpStages) & 1) ^ 1, deadline, sm, p.status)) {
                        raw_extra = 1;  // this chunk's raw copies are in flight, its operand copy is not
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&sm.bfull[o], qb);
                    bulk_g2s(sm.b[o], p.aq + (size_t)kc * p.plan.ppad * QK_K + (size_t)it.p0 * QK_K, qb, &sm.bfull[o]);
                }
                if (!ok) break;
            }
            // drain: every issued copy lands before the CTA can exit
            const uint32_t raw_issued = c + raw_extra, b_issued = c;
            for (uint32_t k = raw_issued > kPfRawStages ? raw_issued - kPfRawStages : 0; k < raw_issued; ++k)
                mbar_wait_bounded(&sm.rfull[k % kPfRawStages], (k / kPfRawStages) & 1, deadline + p.timeout_ns);
            for (uint32_t k = b_issued > kPfOpStages ? b_issued - kPfOpStages : 0; k < b_issued; ++k)
                mbar_wait_bounded(&sm.bfull[k % kPfOpStages], (k / kPfOpStages) & 1, deadline + p.timeout_ns);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer (the warp waits and derives the descriptors; lane 0 issues) ----------------
        uint32_t c = 0;
        bool ok = true;
        for (int item = blockIdx.x; item < total && ok && !pf_aborted(sm); item += gridDim.x) {
            const PfItem it = pf_item(p, sm.tiles, item);
            const int n16 = pad_to(it.nvalid, 16);
            const uint32_t idesc = umma_idesc_i8(kPfMT, n16);
            for (int kc = 0; kc < nkc; ++kc, ++c) {
                const int o = c % kPfOpStages, g = c % kPfGroups;
                if (!pf_wait(&sm.aready[o], (c / kPfOpStages) & 1, deadline, sm, p.status) ||
                    !pf_wait(&sm.bfull[o], (c / kPfOpStages) & 1, deadline, sm, p.status) ||
                    !pf_wait(&sm.gfree[g], ((c / kPfGroups) & 1) ^ 1, deadline, sm, p.status)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t abase = smem_u32(sm.a[o]), bbase = smem_u32(sm.b[o]);
                const uint32_t dbase = tmem + g * kPfGroupCols;
                if (lane == 0) {
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        tc_mma_i8(dbase + j * kPfNT, umma_smem_desc(abase + j * 256, 128, 2048),
                                  umma_smem_desc(bbase + j * 256, 128, 2048), idesc, 1);
                    tc_commit(&sm.gfull[g]);
                    tc_commit(&sm.abempty[o]);
                }
                __syncwarp();
            }
        }
        // all MMAs issued by lane 0 complete before TMEM is released
        if (c > 0 && lane == 0) {
            tc_commit(&sm.mdone);
            mbar_wait_bounded(&sm.mdone, 0, deadline + p.timeout_ns);
        }
        __syncwarp();
    } else if (warp < kPfEpiWarp0) {
        // ---------------- unpack (128 threads, one weight row each) ----------------
        const int t = tid - 64, r = t;
        uint32_t c = 0;
        for (int item = blockIdx.x; item < total && !pf_aborted(sm); item += gridDim.x) {
            const PfItem it = pf_item(p, sm.tiles, item);
            const int n16 = pad_to(it.nvalid, 16);
            bool ok = true;
            for (int kc = 0; kc < nkc; ++kc, ++c) {
                const int s = c % kPfRawStages, o = c % kPfOpStages;
                const uint32_t op = ((c / kPfOpStages) & 1) ^ 1;
                if (!pf_wait(&sm.abempty[o], op, deadline, sm, p.status) ||
                    !pf_wait(&sm.sdempty[o], op, deadline, sm, p.status) ||
                    !pf_wait(&sm.rfull[s], (c / kPfRawStages) & 1, deadline, sm, p.status)) {
                    ok = false;
                    break;
                }
                pf_unpack_row<GT, MODE>(sm.raw[s] + r * bb, sm.a[o], &sm.sc[o][r], r);
                // block scales of the route tile: 16-route records [d8 plane | s8 plane][32-block][16]
                const float *dsraw = reinterpret_cast<const float *>(sm.raw[s] + kPfRawW);
                if (t < n16 * 4) {  // float4 t of the records -> dst[plane][j][route]
                    const int b = t >> 6, plane = (t >> 5) & 1, j = (t >> 2) & 7, c4 = t & 3;
                    *reinterpret_cast<float4 *>(&sm.dst[o][plane][j][b * 16 + c4 * 4]) =
                        *reinterpret_cast<const float4 *>(dsraw + t * 4);
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&sm.rempty[s]);
                    mbar_arrive(&sm.aready[o]);
                }
            }
            if (!ok) break;
        }
    } else {
        // ---------------- epilogue (16 warps) ----------------
        // warp = (TMEM lane quarter qd, route unit u): route columns [8 u, 8 u + 8) of the rows
        // 32 qd .. 32 qd + 31 (units without a route only keep the barriers); per chunk one group
        // wait, then four passes of two 32-blocks.
        const int qd = warp & 3, u = (warp - kPfEpiWarp0) >> 2;
        const int r = qd * 32 + lane;
        const uint32_t tq = tmem + ((uint32_t)(qd * 32) << 16);
        uint32_t c = 0;
        for (int item = blockIdx.x; item < total && !pf_aborted(sm); item += gridDim.x) {
            const PfItem it = pf_item(p, sm.tiles, item);
            const int n16 = pad_to(it.nvalid, 16);
            const bool has = 8 * u < it.nvalid, written = 8 * u < n16;  // read / reset this unit
            float2 acc[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[i] = make_float2(0.0f, 0.0f);
            bool ok = true;
            for (int kc = 0; kc < nkc; ++kc, ++c) {
                const int o = c % kPfOpStages, g = c % kPfGroups;
                if (!pf_wait(&sm.aready[o], (c / kPfOpStages) & 1, deadline, sm, p.status) ||
                    !pf_wait(&sm.gfull[g], (c / kPfGroups) & 1, deadline, sm, p.status)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t gbase = tq + g * kPfGroupCols + 8 * u;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    uint32_t v[8];  // the unit's 8 route columns of 32-block j
                    PfScales8 z;
                    if (has) {
                        // scales first: their shared-memory latency overlaps the TMEM load
                        z = pf_scales8(sm.sc[o][j * kPfMT + r], &sm.dst[o][0][j][8 * u], &sm.dst[o][1][j][8 * u]);
                        tc_ld8(gbase + j * kPfNT, v);
                        tc_wait_ld();
                    }
                    if (written) tc_st8_const(gbase + j * kPfNT, kPfAccBias);
                    if (j == 7) {
                        if (written) tc_wait_st();
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&sm.gfree[g]);  // the group's values are in registers
                    }
                    if (has) pf_accumulate8(acc, v, z);
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&sm.sdempty[o]);
            }
            if (!ok) break;
            const int row = it.m0 + r;
            if (has && row < p.N) {
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int col = 8 * u + i;
                    if (col < it.nvalid) {
                        const int route = p.plan.row_route[it.p0 + col];
                        const float v = (i & 1) ? acc[i >> 1].y : acc[i >> 1].x;
                        p.out[(size_t)route * p.N + row] = p.route_scale ? __fmul_rn(v, p.route_scale[route]) : v;
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kPfTmemCols));
    }
}

// Tensor map over the expert weights viewed as a 2-D array of 32-bit words:
// [E * N rows][row_bytes / 4], box = one super-block (bb / 4 words) x 128 rows.

static int make_weight_map(CUtensorMap *map, const void *w, int gtype, long rows, int K) {
    auto enc = tensor_map_encoder();
    if (!enc) return MMRS_ERR_LAUNCH;
    const int bb = kq_block_bytes(gtype);
    const cuuint64_t row_bytes = (cuuint64_t)(K / QK_K) * bb;
    cuuint64_t dims[2] = {row_bytes / 4, (cuuint64_t)rows};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {(cuuint32_t)(bb / 4), (cuuint32_t)kPfMT};
    cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void *>(w), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? MMRS_OK : MMRS_ERR_ARG;
}

int pf_gemm(const void *weights, PfGemmParams p, int rows_max, cudaStream_t s) {
    (void)rows_max;
    if (p.gtype != MMRS_Q4K && p.gtype != MMRS_Q5K) return MMRS_ERR_UNSUPPORTED;
    if (p.K % QK_K || p.N <= 0 || p.E <= 0 || p.E > kPfMaxExperts) return MMRS_ERR_ARG;
    if (((uintptr_t)weights & 15u) || ((uintptr_t)p.aq & 15u) || ((uintptr_t)p.ads & 15u)) return MMRS_ERR_ARG;
    CUtensorMap map;
    int rc = make_weight_map(&map, weights, p.gtype, (long)p.E * p.N, p.K);
    if (rc != MMRS_OK) return rc;
    p.mt = (p.N + kPfMT - 1) / kPfMT;
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const size_t smem = pf_gemm_smem_bytes();
    static std::once_flag once[64];
    std::call_once(once[dev & 63], [smem] {
        cudaFuncSetAttribute(pf_gemm_kernel<MMRS_Q4K, kPfModeMmq>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        cudaFuncSetAttribute(pf_gemm_kernel<MMRS_Q5K, kPfModeMmq>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        cudaFuncSetAttribute(pf_gemm_kernel<MMRS_Q4K, kPfModeGeneric>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem);
        cudaFuncSetAttribute(pf_gemm_kernel<MMRS_Q5K, kPfModeGeneric>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem);
    });
    const bool mmq = p.mode == kPfModeMmq;
    if (p.gtype == MMRS_Q4K) {
        if (mmq) pf_gemm_kernel<MMRS_Q4K, kPfModeMmq><<<sms, kPfThreads, smem, s>>>(map, p);
        else pf_gemm_kernel<MMRS_Q4K, kPfModeGeneric><<<sms, kPfThreads, smem, s>>>(map, p);
    } else {
        if (mmq) pf_gemm_kernel<MMRS_Q5K, kPfModeMmq><<<sms, kPfThreads, smem, s>>>(map, p);
        else pf_gemm_kernel<MMRS_Q5K, kPfModeGeneric><<<sms, kPfThreads, smem, s>>>(map, p);
    }
    return cudaGetLastError() == cudaSuccess ? MMRS_OK : MMRS_ERR_LAUNCH;
}

}  // namespace mmrs
