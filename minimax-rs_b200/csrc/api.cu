// C ABI entry points: host-side validation, workspace layout and dispatch.
#include <cstddef>
#include <cstdio>
#include <cstring>

#include <algorithm>
#include <mutex>
#include "common.cuh"
#include "decode.cuh"
#include "peer.cuh"
#include "prefill.cuh"
#include "workspace.cuh"

namespace mmrs {

static thread_local int g_last_error = MMRS_OK;
static int set_err(int e) {
    g_last_error = e;
    return e;
}
void record_error(int status) { g_last_error = status; }

// SM count and opt-in shared memory of the current device, queried once per device (they are on
// every call's path; the queries cost more than the rest of the host work of a decode call).
struct DeviceLimits {
    int sms = 0, max_smem = 0;
};
static const DeviceLimits &device_limits() {
    static std::once_flag once[64];
    static DeviceLimits lim[64];
    static DeviceLimits none;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return none;
    std::call_once(once[dev], [dev] {
        cudaDeviceGetAttribute(&lim[dev].sms, cudaDevAttrMultiProcessorCount, dev);
        cudaDeviceGetAttribute(&lim[dev].max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    });
    return lim[dev];
}
static int device_sms() { return device_limits().sms; }
static int device_max_smem() { return device_limits().max_smem; }

static bool aligned16(const void *p) { return ((uintptr_t)p & 15u) == 0; }

// Default bound on any device-side wait: 2 s.
constexpr uint64_t kTimeoutNs = 2000000000ull;

// ------------------------------------------------------------------------------------------
// minimax_moe_decode_topk: one CTA of 256 threads, thread e owns expert e.
// Same arithmetic as minimax_moe_decode_topk_kernel (moe_gguf.cu:34-100): s = 1/(1+expf(-l)),
// stable descending order of s+bias (lower id first on ties, as the stable radix sort),
// weights s/((s0+s4)+(s2+s6))+((s1+s5)+(s3+s7)), then (expert, route) sorted by expert id.
// ------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) decode_topk_kernel(const float *__restrict__ logits,
                                                          const float *__restrict__ bias, uint32_t *topk_ids,
                                                          float *topk_weights, uint32_t *expert_ids,
                                                          uint32_t *route_ids) {
    __shared__ float sel[256];
    __shared__ float sig[256];
    __shared__ int ids[8];
    const int e = threadIdx.x;
    const float sg = __fdiv_rn(1.0f, 1.0f + expf(-logits[e]));
    sig[e] = sg;
    sel[e] = sg + bias[e];
    __syncthreads();
    const float me = sel[e];
    int rank = 0;
#pragma unroll 8
    for (int j = 0; j < 256; ++j) {
        const float o = sel[j];
        rank += (o > me) || (o == me && j < e);
    }
    if (rank < 8) ids[rank] = e;
    __syncthreads();
    if (e == 0) {
        float v[8];
        for (int k = 0; k < 8; ++k) v[k] = sig[ids[k]];
        const float denom = ((v[0] + v[4]) + (v[2] + v[6])) + ((v[1] + v[5]) + (v[3] + v[7]));
        int se[8], sr[8];
        for (int k = 0; k < 8; ++k) {
            topk_ids[k] = (uint32_t)ids[k];
            topk_weights[k] = __fdiv_rn(v[k], denom);
            se[k] = ids[k];
            sr[k] = k;
        }
        for (int i = 1; i < 8; ++i) {
            const int key = se[i], rt = sr[i];
            int j = i - 1;
            while (j >= 0 && se[j] > key) {
                se[j + 1] = se[j];
                sr[j + 1] = sr[j];
                --j;
            }
            se[j + 1] = key;
            sr[j + 1] = rt;
        }
        for (int k = 0; k < 8; ++k) {
            expert_ids[k] = (uint32_t)se[k];
            route_ids[k] = (uint32_t)sr[k];
        }
    }
}

// ------------------------------------------------------------------------------------------
// Workspace layout of the fused block
// ------------------------------------------------------------------------------------------
constexpr int kTraceCtas = 256;
constexpr size_t kTraceOffset = kControlBytes;
static_assert(sizeof(DecodeCtl) <= kControlBytes, "the decode control block lies in the control bytes");
static size_t up256(size_t v) { return (v + 255) / 256 * 256; }
// [control block (DecodeCtl)] | trace | tagged score copies | tagged act records (9 words a Q8_1
// block); all of it zero before first use (the tags of a fresh or reset workspace start again at 1)
WsLayout ws_layout(int E, int I, int max_tokens) {
    (void)E;
    (void)max_tokens;
    WsLayout l;
    const size_t nblk = (size_t)8 * I / 32;
    l.ctl = 0;
    l.trace = kTraceOffset;
    l.score = l.trace + sizeof(uint64_t) * kTraceCtas * kTraceSlots;
    l.arec = l.score + sizeof(unsigned long long) * kScoreReplicas * 256;
    l.total = l.arec + up256(nblk * 9 * sizeof(unsigned long long));
    return l;
}

void ws_bind(DecodeParams &p, uint8_t *ws, const WsLayout &l) {
    p.ctl = reinterpret_cast<DecodeCtl *>(ws + l.ctl);
    p.trace = reinterpret_cast<uint64_t *>(ws + l.trace);
    p.score = reinterpret_cast<unsigned long long *>(ws + l.score);
    p.arec = reinterpret_cast<unsigned long long *>(ws + l.arec);
    p.zero_bytes = (uint32_t)l.total;
}

// ------------------------------------------------------------------------------------------
// Multi-token scratch, placed after the single-token layout in the same workspace.
// ------------------------------------------------------------------------------------------
struct PfLayout {
    size_t logits, ids, wts, skeys, sroutes, count, first, seg, tiles, row_route, aq_h, ads_h, gate, up, aq_i,
        ads_i, dn, total;
    int ppad;
};
static PfLayout pf_layout(size_t base, int E, int H, int I, int T) {
    PfLayout l;
    const size_t M = (size_t)T * 8;
    l.ppad = pf_ppad((int)M, E);
    size_t o = up256(base);
    auto take = [&](size_t bytes) {
        const size_t at = o;
        o = up256(o + bytes);
        return at;
    };
    l.logits = take((size_t)T * E * 4);
    l.ids = take(M * 4);
    l.wts = take(M * 4);
    l.skeys = take(M * 4);
    l.sroutes = take(M * 4);
    l.count = take((size_t)E * 4);
    l.first = take((size_t)E * 4);
    l.seg = take((size_t)E * 4);
    l.tiles = take((size_t)(E + 1) * 4);
    l.row_route = take((size_t)l.ppad * 4);
    l.aq_h = take((size_t)H * l.ppad);
    l.ads_h = take((size_t)(H / 32) * l.ppad * 8);
    l.gate = take(M * I * 4);
    l.up = take(M * I * 4);
    l.aq_i = take((size_t)I * l.ppad);
    l.ads_i = take((size_t)(I / 32) * l.ppad * 8);
    l.dn = take(M * H * 4);
    l.total = o;
    return l;
}
static PfPlan pf_bind_plan(uint8_t *ws, const PfLayout &l) {
    PfPlan p;
    p.count = reinterpret_cast<int *>(ws + l.count);
    p.first = reinterpret_cast<int *>(ws + l.first);
    p.seg = reinterpret_cast<int *>(ws + l.seg);
    p.tiles = reinterpret_cast<int *>(ws + l.tiles);
    p.row_route = reinterpret_cast<int *>(ws + l.row_route);
    p.ppad = l.ppad;
    return p;
}
static int bits_for(int n) {  // smallest b with (n - 1) < 2^b
    int b = 0;
    while ((1 << b) < n) ++b;
    return b;
}

// One routed expert GEMM over scratch it allocates on the stream (the reference's launchers
// also allocate their scratch per call, moe_gguf.cu:381, mmq_moe.cu:105-135).
static int routed_gemm(const float *input, const void *weights, const int32_t *sorted_token_ids,
                       const int32_t *expert_ids, const float *topk_weights, float *output, int num_experts,
                       int topk, int size_m, int size_n, int size_k, int gtype, int mode, cudaStream_t s) {
    if (size_m <= 0) return MMRS_OK;
    if (!input || !weights || !sorted_token_ids || !expert_ids || !output || topk <= 0 || size_n <= 0 ||
        size_k <= 0 || size_k % QK_K || num_experts <= 0)
        return MMRS_ERR_ARG;
    if (gtype != MMRS_Q4K && gtype != MMRS_Q5K) return MMRS_ERR_UNSUPPORTED;
    if (num_experts > kPfMaxExperts) return MMRS_ERR_UNSUPPORTED;
    if (!aligned16(input) || !aligned16(weights)) return MMRS_ERR_ARG;
    const int ppad = pf_ppad(size_m, num_experts);
    size_t o = 0;
    auto take = [&](size_t bytes) {
        const size_t at = o;
        o = up256(o + bytes);
        return at;
    };
    const size_t o_cnt = take((size_t)num_experts * 4), o_first = take((size_t)num_experts * 4),
                 o_seg = take((size_t)num_experts * 4), o_tiles = take((size_t)(num_experts + 1) * 4),
                 o_rr = take((size_t)ppad * 4), o_q = take((size_t)size_k * ppad),
                 o_ds = take((size_t)(size_k / 32) * ppad * 8), o_st = take(256);
    uint8_t *ws = nullptr;
    if (cudaMallocAsync((void **)&ws, o, s) != cudaSuccess) return MMRS_ERR_ALLOC;
    cudaMemsetAsync(ws + o_st, 0, 4, s);
    PfPlan plan;
    plan.count = reinterpret_cast<int *>(ws + o_cnt);
    plan.first = reinterpret_cast<int *>(ws + o_first);
    plan.seg = reinterpret_cast<int *>(ws + o_seg);
    plan.tiles = reinterpret_cast<int *>(ws + o_tiles);
    plan.row_route = reinterpret_cast<int *>(ws + o_rr);
    plan.ppad = ppad;
    PfActs acts{reinterpret_cast<int8_t *>(ws + o_q), reinterpret_cast<float *>(ws + o_ds)};
    int rc = pf_build_plan(expert_ids, sorted_token_ids, size_m, num_experts, plan, s);
    if (rc == MMRS_OK)
        rc = pf_quantize(input, nullptr, topk_weights ? 1 : topk, size_k, mode, plan, acts, ppad, s);
    if (rc == MMRS_OK) {
        PfGemmParams g = {};
        g.aq = acts.q;
        g.ads = acts.ds;
        g.plan = plan;
        g.route_scale = topk_weights;
        g.out = output;
        g.E = num_experts;
        g.N = size_n;
        g.K = size_k;
        g.gtype = gtype;
        g.mode = mode;
        g.status = reinterpret_cast<uint32_t *>(ws + o_st);
        g.timeout_ns = kTimeoutNs;
        rc = pf_gemm(weights, g, ppad, s);
    }
    cudaFreeAsync(ws, s);
    return rc;
}

int validate_weights(const MmrsMoeWeights *w) {
    if (!w || !w->router || !w->bias || !w->gate || !w->up || !w->down) return MMRS_ERR_ARG;
    if (w->hidden <= 0 || w->inter <= 0 || w->hidden % QK_K || w->inter % QK_K) return MMRS_ERR_ARG;
    if ((w->gate_up_type != MMRS_Q4K && w->gate_up_type != MMRS_Q5K) ||
        (w->down_type != MMRS_Q4K && w->down_type != MMRS_Q5K))
        return MMRS_ERR_UNSUPPORTED;
    if (w->topk != 8 || w->num_experts < 8 || w->num_experts > 1024) return MMRS_ERR_UNSUPPORTED;
    if (!aligned16(w->gate) || !aligned16(w->up) || !aligned16(w->down) || !aligned16(w->router))
        return MMRS_ERR_ARG;
    return MMRS_OK;
}

}  // namespace mmrs

using namespace mmrs;

extern "C" int mmrs_last_error(void) { return g_last_error; }

extern "C" void minimax_moe_decode_topk(const float *logits, const float *bias, uint32_t *topk_ids,
                                        float *topk_weights, uint32_t *expert_ids, uint32_t *route_ids,
                                        mmrs_stream_t stream) {
    if (!logits || !bias || !topk_ids || !topk_weights || !expert_ids || !route_ids) {
        set_err(MMRS_ERR_ARG);
        return;
    }
    decode_topk_kernel<<<1, 256, 0, (cudaStream_t)stream>>>(logits, bias, topk_ids, topk_weights, expert_ids,
                                                            route_ids);
    set_err(cudaGetLastError() == cudaSuccess ? MMRS_OK : MMRS_ERR_LAUNCH);
}

extern "C" void moe_gemm_gguf_decode_silu(const float *input, const void *gate_weights, const void *up_weights,
                                          const void *down_weights, const int32_t *sorted_token_ids,
                                          const int32_t *expert_ids, const float *topk_weights, float *output,
                                          int num_experts, int topk, int hidden_size, int intermediate_size,
                                          int gate_up_gguf_dtype, int down_gguf_dtype, mmrs_stream_t stream) {
    // The reference returns without work for topk != 8 (moe_gguf.cu:457-459); so does this path,
    // but it records the condition.
    if (topk != 8) {
        set_err(MMRS_ERR_UNSUPPORTED);
        return;
    }
    if (!input || !gate_weights || !up_weights || !down_weights || !sorted_token_ids || !expert_ids ||
        !topk_weights || !output || hidden_size <= 0 || intermediate_size <= 0) {
        set_err(MMRS_ERR_ARG);
        return;
    }
    if (!aligned16(gate_weights) || !aligned16(up_weights) || !aligned16(down_weights) || !aligned16(input)) {
        set_err(MMRS_ERR_ARG);
        return;
    }
    DecodeParams p = {};
    p.x = input;
    p.gate = (const uint8_t *)gate_weights;
    p.up = (const uint8_t *)up_weights;
    p.down = (const uint8_t *)down_weights;
    p.y = output;
    p.ext_route = sorted_token_ids;
    p.ext_expert = expert_ids;
    p.ext_w = topk_weights;
    p.internal_routing = 0;
    p.E = num_experts;
    p.H = hidden_size;
    p.I = intermediate_size;
    p.gu_type = gate_up_gguf_dtype;
    p.dn_type = down_gguf_dtype;
    p.timeout_ns = kTimeoutNs;
    int rc = decode_configure(p, device_sms(), device_max_smem());
    if (rc != MMRS_OK) {
        set_err(rc);
        return;
    }
    // Scratch on the stream's pool, like the reference (moe_gguf.cu:468-472).
    const WsLayout l = ws_layout(num_experts, intermediate_size, 1);
    cudaStream_t s = (cudaStream_t)stream;
    uint8_t *ws = nullptr;
    if (cudaMallocAsync((void **)&ws, l.total, s) != cudaSuccess) {
        set_err(MMRS_ERR_ALLOC);
        return;
    }
    cudaMemsetAsync(ws, 0, l.total, s);
    ws_bind(p, ws, l);
    p.trace = nullptr;
    rc = decode_launch(p, s);
    cudaFreeAsync(ws, s);
    set_err(rc);
}

extern "C" void moe_gemm_gguf(const float *input, const void *weights, const int32_t *sorted_token_ids,
                              const int32_t *expert_ids, const float *topk_weights, float *output, int num_experts,
                              int topk, int size_m, int size_n, int size_k, int gguf_dtype, mmrs_stream_t stream) {
    set_err(routed_gemm(input, weights, sorted_token_ids, expert_ids, topk_weights, output, num_experts, topk,
                        size_m, size_n, size_k, gguf_dtype, kPfModeGeneric, (cudaStream_t)stream));
}

extern "C" void moe_gemm_mmq_gguf(const float *input, const void *weights, const int32_t *sorted_token_ids,
                                  const int32_t *expert_ids, const float *topk_weights, float *output,
                                  int num_experts, int topk, int size_m, int size_n, int size_k, int gguf_dtype,
                                  mmrs_stream_t stream) {
    // Like the reference (mmq_moe.cu:84-86) types other than Q4_K / Q5_K do nothing; the
    // condition is recorded for mmrs_last_error().
    set_err(routed_gemm(input, weights, sorted_token_ids, expert_ids, topk_weights, output, num_experts, topk,
                        size_m, size_n, size_k, gguf_dtype, kPfModeMmq, (cudaStream_t)stream));
}

extern "C" void moe_sort_routes(const uint32_t *expert_ids_unsorted, uint32_t *expert_ids_sorted,
                                uint32_t *route_ids_sorted, int size, int end_bit, mmrs_stream_t stream) {
    if (size > 0 && (!expert_ids_unsorted || !expert_ids_sorted || !route_ids_sorted)) {
        set_err(MMRS_ERR_ARG);
        return;
    }
    set_err(pf_sort_routes(expert_ids_unsorted, size, end_bit, expert_ids_sorted, route_ids_sorted,
                           (cudaStream_t)stream));
}

extern "C" size_t mmrs_moe_workspace_zero_bytes(const MmrsMoeWeights *w) {
    return w ? ws_layout(w->num_experts, w->inter, 1).total : 0;
}

extern "C" size_t mmrs_moe_workspace_bytes(const MmrsMoeWeights *w, int max_tokens) {
    if (!w) return 0;
    const size_t single = ws_layout(w->num_experts, w->inter, 1).total;
    if (max_tokens <= 1) return single;
    return pf_layout(single, w->num_experts, w->hidden, w->inter, max_tokens).total;
}

// T > 1: router GEMM, top-8, stable bucketing, gathered Q8_1 (MMQ numerics for T >= 32, the
// generic ones below, as fused_moe.rs:296-316 selects), gate / up GEMMs, SiLU * up fused into
// the down operand's quantisation, down GEMM scaled by the route weight, top-8 sum + residual.
static int block_forward_multi(const MmrsMoeWeights *w, const float *x, const float *residual, float *y, int T,
                               uint32_t *topk_ids, float *topk_weights, uint8_t *ws, cudaStream_t s,
                               int own_world = 1, int own_rank = 0) {
    const int E = w->num_experts, H = w->hidden, I = w->inter, M = T * 8;
    const PfLayout l = pf_layout(ws_layout(E, I, 1).total, E, H, I, T);
    float *logits = reinterpret_cast<float *>(ws + l.logits);
    uint32_t *ids = topk_ids ? topk_ids : reinterpret_cast<uint32_t *>(ws + l.ids);
    float *wts = topk_weights ? topk_weights : reinterpret_cast<float *>(ws + l.wts);
    uint32_t *skeys = reinterpret_cast<uint32_t *>(ws + l.skeys), *sroutes = reinterpret_cast<uint32_t *>(ws + l.sroutes);
    const PfPlan plan = pf_bind_plan(ws, l);
    const PfActs xh{reinterpret_cast<int8_t *>(ws + l.aq_h), reinterpret_cast<float *>(ws + l.ads_h)};
    const PfActs xi{reinterpret_cast<int8_t *>(ws + l.aq_i), reinterpret_cast<float *>(ws + l.ads_i)};
    float *g = reinterpret_cast<float *>(ws + l.gate), *u = reinterpret_cast<float *>(ws + l.up);
    float *dn = reinterpret_cast<float *>(ws + l.dn);
    const int mode_gu = T >= 32 ? kPfModeMmq : kPfModeGeneric;
    const int mode_dn = T >= 32 ? kPfModeMmq : kPfModeGeneric;
    uint32_t *status = reinterpret_cast<uint32_t *>(ws);  // workspace status word

    int rc = pf_router_logits(x, w->router, T, E, H, logits, s);
    if (rc == MMRS_OK) rc = pf_route_topk(logits, w->bias, T, E, ids, wts, s);
    if (rc == MMRS_OK) rc = pf_sort_routes(ids, M, bits_for(E), skeys, sroutes, s);
    if (rc == MMRS_OK)
        rc = pf_build_plan(reinterpret_cast<const int32_t *>(skeys), reinterpret_cast<const int32_t *>(sroutes), M, E,
                           plan, s, own_world, own_rank);
    if (rc == MMRS_OK) rc = pf_quantize(x, nullptr, 8, H, mode_gu, plan, xh, l.ppad, s);
    PfGemmParams gp = {};
    gp.plan = plan;
    gp.E = E;
    gp.status = status;
    gp.timeout_ns = kTimeoutNs;
    if (rc == MMRS_OK) {
        gp.aq = xh.q;
        gp.ads = xh.ds;
        gp.N = I;
        gp.K = H;
        gp.gtype = w->gate_up_type;
        gp.mode = mode_gu;
        gp.out = g;
        rc = pf_gemm(w->gate, gp, l.ppad, s);
        if (rc == MMRS_OK) {
            gp.out = u;
            rc = pf_gemm(w->up, gp, l.ppad, s);
        }
    }
    if (rc == MMRS_OK) rc = pf_quantize(g, u, 1, I, mode_dn, plan, xi, l.ppad, s);
    if (rc == MMRS_OK) {
        gp.aq = xi.q;
        gp.ads = xi.ds;
        gp.N = H;
        gp.K = I;
        gp.gtype = w->down_type;
        gp.mode = mode_dn;
        gp.route_scale = wts;
        gp.out = dn;
        rc = pf_gemm(w->down, gp, l.ppad, s);
    }
    if (rc == MMRS_OK) rc = pf_reduce_topk(dn, residual, T, H, y, s, ids, own_world, own_rank);
    return rc;
}

extern "C" int mmrs_moe_block_forward(const MmrsMoeWeights *w, const float *x, const float *residual, float *y,
                                      int num_tokens, uint32_t *topk_ids, float *topk_weights, void *workspace,
                                      size_t workspace_bytes, mmrs_stream_t stream) {
    int rc = validate_weights(w);
    if (rc != MMRS_OK) return rc;
    if (!x || !y || num_tokens < 0 || !workspace) return MMRS_ERR_ARG;
    if (num_tokens == 0) return MMRS_OK;
    const WsLayout l = ws_layout(w->num_experts, w->inter, 1);
    if (workspace_bytes < mmrs_moe_workspace_bytes(w, num_tokens) || !aligned16(workspace) || !aligned16(x) ||
        !aligned16(y) || (residual && !aligned16(residual)))
        return MMRS_ERR_ARG;
    uint8_t *ws = (uint8_t *)workspace;
    if (num_tokens > 1) return block_forward_multi(w, x, residual, y, num_tokens, topk_ids, topk_weights, ws,
                                                   (cudaStream_t)stream);
    DecodeParams p = {};
    p.x = x;
    p.router = w->router;
    p.bias = w->bias;
    p.gate = (const uint8_t *)w->gate;
    p.up = (const uint8_t *)w->up;
    p.down = (const uint8_t *)w->down;
    p.residual = residual;
    p.y = y;
    p.topk_ids_out = topk_ids;
    p.topk_w_out = topk_weights;
    p.internal_routing = 1;
    ws_bind(p, ws, l);
    p.E = w->num_experts;
    p.H = w->hidden;
    p.I = w->inter;
    p.gu_type = w->gate_up_type;
    p.dn_type = w->down_type;
    p.timeout_ns = kTimeoutNs;
    rc = decode_configure(p, device_sms(), device_max_smem());
    if (rc != MMRS_OK) return rc;
    return decode_launch(p, (cudaStream_t)stream);
}

// Device view of pinned host memory (UVA), or null when the memory is not mapped (the failed
// query's error is cleared so that later launch checks do not see it).
static void *mapped_host(const void *h) {
    void *d = nullptr;
    if (cudaHostGetDevicePointer(&d, const_cast<void *>(h), 0) == cudaSuccess) return d;
    (void)cudaGetLastError();
    return nullptr;
}

// Reads n floats (n % 4 == 0, 16-byte aligned) from mapped host memory into device memory:
// for small messages the loads' PCIe round trip is shorter than a copy-engine transfer.
__global__ void __launch_bounds__(256) host_in_kernel(const float4 *__restrict__ src, float4 *__restrict__ dst,
                                                      size_t n4) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x)
        dst[i] = src[i];
}

// n floats of x from host memory into x_dev on `s`: loads from the mapped pinned buffer by a small
// kernel (the next launch then follows it on the device at once), else a copy-engine transfer.
static int host_input(const float *x_host, float *x_dev, size_t n, cudaStream_t s) {
    const void *xm = aligned16(x_host) ? mapped_host(x_host) : nullptr;
    if (xm) {
        const size_t n4 = n / 4;  // hidden is a multiple of 256
        const unsigned blocks = (unsigned)std::min<size_t>((n4 + 255) / 256, 1184);
        host_in_kernel<<<blocks, 256, 0, s>>>(reinterpret_cast<const float4 *>(xm), reinterpret_cast<float4 *>(x_dev), n4);
        return cudaGetLastError() == cudaSuccess ? MMRS_OK : MMRS_ERR_LAUNCH;
    }
    return cudaMemcpyAsync(x_dev, x_host, n * sizeof(float), cudaMemcpyHostToDevice, s) == cudaSuccess
               ? MMRS_OK
               : MMRS_ERR_LAUNCH;
}

extern "C" int mmrs_moe_block_forward_host(const MmrsMoeWeights *w, const float *x_host, const float *residual,
                                           float *y_host, int num_tokens, float *x_dev, float *y_dev,
                                           uint32_t *topk_ids, float *topk_weights, void *workspace,
                                           size_t workspace_bytes, mmrs_stream_t stream) {
    int rc = validate_weights(w);
    if (rc != MMRS_OK) return rc;
    if (!x_host || !y_host || !x_dev || !y_dev || num_tokens < 0) return MMRS_ERR_ARG;
    if (num_tokens == 0) return MMRS_OK;
    const size_t n = (size_t)num_tokens * w->hidden;
    cudaStream_t s = (cudaStream_t)stream;
    rc = host_input(x_host, x_dev, n, s);
    if (rc != MMRS_OK) return rc;
    // output: the block's final stores go straight to the mapped pinned buffer, else via y_dev
    void *ym = aligned16(y_host) ? mapped_host(y_host) : nullptr;
    rc = mmrs_moe_block_forward(w, x_dev, residual, ym ? static_cast<float *>(ym) : y_dev, num_tokens, topk_ids,
                                topk_weights, workspace, workspace_bytes, stream);
    if (rc != MMRS_OK || ym) return rc;
    return cudaMemcpyAsync(y_host, y_dev, n * sizeof(float), cudaMemcpyDeviceToHost, s) == cudaSuccess ? MMRS_OK
                                                                                                      : MMRS_ERR_LAUNCH;
}

extern "C" int mmrs_moe_workspace_status(void *workspace, mmrs_stream_t stream) {
    if (!workspace) return MMRS_ERR_ARG;
    uint32_t status = 0;
    cudaStream_t s = (cudaStream_t)stream;
    if (cudaMemcpyAsync(&status, workspace, sizeof(status), cudaMemcpyDeviceToHost, s) != cudaSuccess)
        return MMRS_ERR_LAUNCH;
    if (cudaStreamSynchronize(s) != cudaSuccess) return MMRS_ERR_LAUNCH;
    if (status != 0) {
        // reset the zeroed prefix (control block, trace, tagged records: its size is kept in the
        // control block by the kernel) so the workspace is usable again
        uint32_t zero = 0;
        cudaMemcpyAsync(&zero, (const uint8_t *)workspace + offsetof(DecodeCtl, zero_bytes), sizeof(zero),
                        cudaMemcpyDeviceToHost, s);
        cudaStreamSynchronize(s);
        cudaMemsetAsync(workspace, 0, zero > kControlBytes ? zero : kControlBytes, s);
        cudaStreamSynchronize(s);
    }
    return (int)status;
}

extern "C" int mmrs_moe_workspace_trace(const void *workspace, uint64_t *host_out, int max_entries,
                                        mmrs_stream_t stream) {
    if (!workspace || !host_out || max_entries <= 0) return -MMRS_ERR_ARG;
    const int n = max_entries < kTraceCtas * kTraceSlots ? max_entries : kTraceCtas * kTraceSlots;
    cudaStream_t s = (cudaStream_t)stream;
    if (cudaMemcpyAsync(host_out, (const uint8_t *)workspace + kTraceOffset, sizeof(uint64_t) * n,
                        cudaMemcpyDeviceToHost,
                        s) != cudaSuccess)
        return -MMRS_ERR_LAUNCH;
    if (cudaStreamSynchronize(s) != cudaSuccess) return -MMRS_ERR_LAUNCH;
    return n;
}

extern "C" int mmrs_moe_block_forward_group(const MmrsMoeWeights *w, const MmrsPeerGroup *g, const float *x,
                                            const float *residual, float *y, int num_tokens, uint32_t *topk_ids,
                                            float *topk_weights, void *workspace, size_t workspace_bytes,
                                            uint32_t token, mmrs_stream_t stream) {
    if (!g || g->world < 1 || g->world > kMaxRanks || g->rank < 0 || g->rank >= g->world) return MMRS_ERR_ARG;
    if (g->world == 1)
        return mmrs_moe_block_forward(w, x, residual, y, num_tokens, topk_ids, topk_weights, workspace,
                                      workspace_bytes, stream);
    int rc = validate_weights(w);
    if (rc != MMRS_OK) return rc;
    if (!x || !y || num_tokens < 0 || !workspace || !g->mine) return MMRS_ERR_ARG;
    for (int r = 0; r < g->world; ++r)
        if (!g->peers[r]) return MMRS_ERR_ARG;
    if (num_tokens == 0) return MMRS_OK;
    if (workspace_bytes < mmrs_moe_workspace_bytes(w, num_tokens) || !aligned16(workspace) || !aligned16(x) ||
        !aligned16(y) || (residual && !aligned16(residual)))
        return MMRS_ERR_ARG;
    if (w->hidden > kXchMaxHidden) return MMRS_ERR_UNSUPPORTED;
    if (token == 0) return MMRS_ERR_ARG;  // tokens start at 1 (flags are zero-initialised)
    uint8_t *ws = (uint8_t *)workspace;
    cudaStream_t s = (cudaStream_t)stream;
    const int ep = g->expert_parallel ? 1 : 0;
    if (num_tokens > 1) {
        // rank-local block into this rank's all-reduce buffer, then the peer all-reduce (+ residual)
        const size_t count = (size_t)num_tokens * w->hidden;
        if (count > g->ar_capacity) return MMRS_ERR_ARG;
        float *partial = mmrs_xch_ar_buffer(g, token);
        rc = block_forward_multi(w, x, nullptr, partial, num_tokens, topk_ids, topk_weights, ws, s,
                                 ep ? g->world : 1, ep ? g->rank : 0);
        if (rc != MMRS_OK) return rc;
        return mmrs_peer_all_reduce(g, residual, y, count, token, stream);
    }
    const WsLayout l = ws_layout(w->num_experts, w->inter, 1);
    DecodeParams p = {};
    p.x = x;
    p.router = w->router;
    p.bias = w->bias;
    p.gate = (const uint8_t *)w->gate;
    p.up = (const uint8_t *)w->up;
    p.down = (const uint8_t *)w->down;
    p.residual = residual;
    p.y = y;
    p.topk_ids_out = topk_ids;
    p.topk_w_out = topk_weights;
    p.internal_routing = 1;
    ws_bind(p, ws, l);
    p.E = w->num_experts;
    p.H = w->hidden;
    p.I = w->inter;
    p.gu_type = w->gate_up_type;
    p.dn_type = w->down_type;
    p.timeout_ns = kTimeoutNs;
    p.xch = static_cast<uint8_t *>(g->mine);
    for (int r = 0; r < g->world; ++r) p.xpeer[r] = static_cast<uint8_t *>(g->peers[r]);
    p.world = g->world;
    p.rank = g->rank;
    p.ep = ep;
    p.token = token;
    rc = decode_configure(p, device_sms(), device_max_smem());
    if (rc != MMRS_OK) return rc;
    return decode_launch(p, s);
}

extern "C" int mmrs_moe_block_forward_group_host(const MmrsMoeWeights *w, const MmrsPeerGroup *g, const float *x_host,
                                                 const float *residual, float *y_host, int num_tokens, float *x_dev,
                                                 float *y_dev, uint32_t *topk_ids, float *topk_weights,
                                                 void *workspace, size_t workspace_bytes, uint32_t token,
                                                 mmrs_stream_t stream) {
    int rc = validate_weights(w);
    if (rc != MMRS_OK) return rc;
    if (!g || !x_host || !y_host || !x_dev || !y_dev || num_tokens < 0) return MMRS_ERR_ARG;
    if (num_tokens == 0) return MMRS_OK;
    const size_t n = (size_t)num_tokens * w->hidden;
    cudaStream_t s = (cudaStream_t)stream;
    rc = host_input(x_host, x_dev, n, s);
    if (rc != MMRS_OK) return rc;
    // output: the group's final stores (the decode kernel's rank-ordered sums, or the peer
    // all-reduce) go straight to the mapped pinned buffer, else via y_dev
    void *ym = aligned16(y_host) ? mapped_host(y_host) : nullptr;
    rc = mmrs_moe_block_forward_group(w, g, x_dev, residual, ym ? static_cast<float *>(ym) : y_dev, num_tokens, topk_ids,
                                      topk_weights, workspace, workspace_bytes, token, stream);
    if (rc != MMRS_OK || ym) return rc;
    return cudaMemcpyAsync(y_host, y_dev, n * sizeof(float), cudaMemcpyDeviceToHost, s) == cudaSuccess ? MMRS_OK
                                                                                                      : MMRS_ERR_LAUNCH;
}
