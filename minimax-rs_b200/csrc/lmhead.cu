// Output projection (LM head) of a MiniMax-M2.7 decode step on B200 (sm_100a): the Q6_K
// `output` matrix (vocabulary x hidden) against the final hidden state, with the greedy token.
//
// Reference path (minimax-rs, src/tensor_parallel_model.rs:871-880, src/sampling.rs:84-88):
// output_norm (candle-nn RmsNorm) -> QMatMul (quantize_q8_1 + mmvq q6_k, mmvq_gguf.cu:384-400,
// 609-632, 808-809) -> argmax of the logits.
//
// HBM-bound (504 MB of Q6_K weights per token at the model's 200064 x 3072), so one streaming
// kernel: one CTA per SM owns a contiguous range of rows (even-aligned: a Q6_K row is 2520
// bytes, 16-byte aligned every second row), streamed in groups of 6 rows through a ring of 12
// shared-memory slots by bulk copies from a producer warp; 11 consumer warps take a group at a
// time with lane = the reference's iqs (8 of a super-block's 256 weights) and three rows a step,
// the lane's Q8_1 activation words in registers.  Logits go to global memory; each CTA
// folds its best (value, lowest index) into one 64-bit atomic maximum and the last CTA to finish
// writes the token.
#include <cuda_fp16.h>

#include <algorithm>
#include <mutex>

#include "../../include/minimax_lmhead.h"
#include "common.cuh"
#include "tma.cuh"
#include "workspace.cuh"

namespace mmrs {

constexpr int kQ6Bytes = 210;       // ql[128] | qh[64] | int8 scales[16] | half d
// 11 consumer warps + the producer = 12 warps, 3 per scheduler: 168 registers a thread are
// available (144 used), enough for three rows in flight per warp; 17 warps capped the kernel at
// 96 registers (measured 101 us per token against 129 us at 16 warps x 2 rows).
constexpr int kLmConsumers = 11;
constexpr int kLmThreads = 32 * (kLmConsumers + 1);
constexpr int kLmSlots = 12;
constexpr int kLmSlotBytes = 16384;
constexpr int kLmGroupRows = 6;     // 15120 bytes: a multiple of 16
constexpr int kLmRowsPerStep = 3;   // independent rows per warp step
constexpr int kLmMaxK = 8192;
constexpr int kLmMaxGroups = 512;

struct LmParams {
    const uint8_t *w;   // Q6_K [rows][k / 256 x 210 B]
    int rows, k;
    const uint8_t *vy;  // Q8_1 activation [k / 32 x 36 B], 16-byte aligned
    float *logits;      // [rows]
    int32_t *token;     // greedy token (null: logits only)
    unsigned long long *best;  // packed (ordered value, ~index) maximum, zero before first use
    uint32_t *ticket;   // CTAs done, zero before first use (both left zero)
    uint32_t *status;   // optional: MMRS_ERR_TIMEOUT when a wait expired
};


// 32-bit word at byte offset `off` (2-byte aligned) of a row in shared memory.
__device__ __forceinline__ uint32_t lm_word(const uint8_t *row, int off) {
    const uint32_t *w = reinterpret_cast<const uint32_t *>(row + (off & ~3));
    return (off & 3) ? __funnelshift_r(w[0], w[1], 16) : w[0];
}

// R rows: lane = iqs.  Per super-block, the lane's 4 low-nibble and 4 high-nibble weights
// (vl, vh as vec_dot_q6_K_q8_1 reads them) as signed bytes q - 32 (per byte (q + 0x60) ^ 0x80:
// q <= 63, so no carry crosses a byte), dotted with the lane's two activation words u[s][i],
// scaled by the 16-weight scales and the activation block scales d8, then by the super-block d:
// the reference's d * (d8[0] * (dot0 * sc0) + d8[1] * (dot1 * sc1)) summed over the row, then the
// warp butterfly.  The R rows are independent chains (more loads in flight per warp).
template <int NSB, int R>
__device__ __forceinline__ void lm_rows_dot(const uint8_t *rows, size_t row_bytes, int lane, const int (&u)[NSB][2],
                                            const float (&d8)[NSB][2], float (&out)[R]) {
    const int qh_word = (lane / 16) * 8 + lane % 8, vh_shift = 2 * ((lane % 16) / 8);
    const int so = (lane / 16) * 8 + (lane % 16) / 4;
#pragma unroll
    for (int q = 0; q < R; ++q) out[q] = 0.0f;
#pragma unroll
    for (int s = 0; s < NSB; ++s) {
#pragma unroll
        for (int q = 0; q < R; ++q) {
            const uint8_t *row = rows + q * row_bytes;
            const int base = s * kQ6Bytes;
            const uint32_t vl = lm_word(row, base + 4 * lane);
            const uint32_t vh = lm_word(row, base + 128 + 4 * qh_word) >> vh_shift;
            const int sc0 = (int8_t)row[base + 192 + so], sc1 = (int8_t)row[base + 192 + so + 4];
            const float d = __half2float(*reinterpret_cast<const __half *>(row + base + 208));
            const uint32_t v0 = (((vl & 0x0F0F0F0Fu) | ((vh << 4) & 0x30303030u)) + 0x60606060u) ^ 0x80808080u;
            const uint32_t v1 = ((((vl >> 4) & 0x0F0F0F0Fu) | (vh & 0x30303030u)) + 0x60606060u) ^ 0x80808080u;
            const int dot0 = __dp4a((int)v0, u[s][0], 0), dot1 = __dp4a((int)v1, u[s][1], 0);
            // |dot * sc| < 2^20: exact conversion on the integer / FP32 pipes (int22_to_float)
            float sumf = 0.0f;
            sumf += d8[s][0] * int22_to_float(dot0 * sc0);
            sumf += d8[s][1] * int22_to_float(dot1 * sc1);
            out[q] += d * sumf;
        }
    }
#pragma unroll
    for (int m = 16; m > 0; m >>= 1)
#pragma unroll
        for (int q = 0; q < R; ++q) out[q] += __shfl_xor_sync(0xffffffffu, out[q], m);
}

template <int NSB>
__global__ void __launch_bounds__(kLmThreads, 1) lm_q6k_kernel(const LmParams p) {
    extern __shared__ __align__(128) uint8_t lm_smem[];
    uint8_t *slots = lm_smem;
    uint8_t *act = slots + (size_t)kLmSlots * kLmSlotBytes;
    uint64_t *full = reinterpret_cast<uint64_t *>(act + kLmMaxK / 32 * 36);
    uint64_t *empty = full + kLmSlots;
    uint64_t *abar = empty + kLmSlots;
    unsigned long long *wbest = reinterpret_cast<unsigned long long *>(abar + 1);  // [kLmConsumers]
    int *ticket = reinterpret_cast<int *>(wbest + kLmConsumers);                 // [kLmSlots]
    int *flag = ticket + kLmSlots;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const size_t row_bytes = (size_t)NSB * kQ6Bytes;
    // even-aligned contiguous row range; an odd last row of the matrix is read from global memory
    const int pairs = p.rows / 2;
    const int r0 = 2 * (int)((long)blockIdx.x * pairs / gridDim.x);
    const int r1 = 2 * (int)((long)(blockIdx.x + 1) * pairs / gridDim.x);
    const int ng = (r1 - r0 + kLmGroupRows - 1) / kLmGroupRows;
    const uint64_t deadline = globaltimer_ns() + 2000000000ull;
    auto issue = [&](int j) {
        const int st = j % kLmSlots, g0 = r0 + j * kLmGroupRows, n = min(kLmGroupRows, r1 - g0);
        const uint32_t bytes = (uint32_t)(n * row_bytes);
        *reinterpret_cast<volatile int *>(&ticket[st]) = j;
        mbar_arrive_expect_tx(&full[st], bytes);
        bulk_g2s(slots + (size_t)st * kLmSlotBytes, p.w + (size_t)g0 * row_bytes, bytes, &full[st]);
    };
    if (threadIdx.x == kLmConsumers * 32) {
        for (int i = 0; i < kLmSlots; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
            ticket[i] = -1;
        }
        mbar_init(abar, 1);
        fence_mbar_init();
        for (int j = 0; j < ng && j < kLmSlots; ++j) issue(j);  // weights: independent of the previous kernel
    }
    __syncthreads();
    grid_dependency_wait();
    launch_dependents();
    const int nb = p.k / 32;
    if (warp == kLmConsumers) {  // producer: the activation, then refills as groups are consumed
        if (lane == 0) {
            mbar_arrive_expect_tx(abar, (uint32_t)(nb * 36));
            bulk_g2s(act, p.vy, (uint32_t)(nb * 36), abar);
            for (int j = kLmSlots; j < ng; ++j) {
                const int st = j % kLmSlots;
                if (!mbar_wait_sleep(&empty[st], (uint32_t)(((j / kLmSlots) - 1) & 1), deadline)) {
                    if (p.status) atomicExch(p.status, (uint32_t)MMRS_ERR_TIMEOUT);
                    break;
                }
                issue(j);
            }
        }
        return;
    }
    bool ok = mbar_wait_sleep(abar, 0u, deadline);
    // the lane's activation words: super-block s, part i -> Q8_1 block 8s + bq8_offset + 2i
    int u[NSB][2];
    float d8[NSB][2];
    {
        const int bq8 = 4 * (lane / 16) + (lane % 16) / 8;
#pragma unroll
        for (int s = 0; s < NSB; ++s)
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const uint8_t *blk = act + (size_t)(8 * s + bq8 + 2 * i) * 36;
                u[s][i] = reinterpret_cast<const int *>(blk + 4)[lane % 8];
                d8[s][i] = __half2float(*reinterpret_cast<const __half *>(blk));
            }
    }
    unsigned long long best = 0ull;
    for (int j = warp; j < ng && ok; j += kLmConsumers) {
        const int st = j % kLmSlots;
        if (!ring_wait(full, ticket, st, j, kLmSlots, deadline)) {
            ok = false;
            break;
        }
        const uint8_t *g = slots + (size_t)st * kLmSlotBytes;
        const int g0 = r0 + j * kLmGroupRows, n = min(kLmGroupRows, r1 - g0);
        int i = 0;
        for (; i + kLmRowsPerStep <= n; i += kLmRowsPerStep) {
            float v[kLmRowsPerStep];
            lm_rows_dot<NSB, kLmRowsPerStep>(g + (size_t)i * row_bytes, row_bytes, lane, u, d8, v);
            if (lane == 0) {
#pragma unroll
                for (int q = 0; q < kLmRowsPerStep; ++q) {
                    p.logits[g0 + i + q] = v[q];
                    const unsigned long long key = lm_key(v[q], g0 + i + q);
                    best = key > best ? key : best;
                }
            }
        }
        for (; i < n; ++i) {  // the last group of a CTA may be shorter
            float v[1];
            lm_rows_dot<NSB, 1>(g + (size_t)i * row_bytes, row_bytes, lane, u, d8, v);
            if (lane == 0) {
                p.logits[g0 + i] = v[0];
                const unsigned long long key = lm_key(v[0], g0 + i);
                best = key > best ? key : best;
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
    }
    if (ok && (p.rows & 1) && blockIdx.x == gridDim.x - 1 && warp == 0) {  // odd last row, from global memory
        const int r = p.rows - 1;
        float v[1];
        lm_rows_dot<NSB, 1>(p.w + (size_t)r * row_bytes, row_bytes, lane, u, d8, v);
        if (lane == 0) {
            p.logits[r] = v[0];
            const unsigned long long key = lm_key(v[0], r);
            best = key > best ? key : best;
        }
    }
    if (!ok && lane == 0 && p.status) atomicExch(p.status, (uint32_t)MMRS_ERR_TIMEOUT);
    if (!p.token) return;
    // greedy token: warp bests -> one atomic maximum per CTA -> the last CTA writes the token
    if (lane == 0) wbest[warp] = best;
    named_sync(1, kLmConsumers * 32);
    if (threadIdx.x == 0) {
        unsigned long long b = 0ull;
        for (int w = 0; w < kLmConsumers; ++w) b = wbest[w] > b ? wbest[w] : b;
        atomicMax(p.best, b);
        __threadfence();
        *flag = atomicAdd(p.ticket, 1u) == gridDim.x - 1;
        if (*flag) {
            __threadfence();
            const unsigned long long k = atomicExch(p.best, 0ull);
            *p.token = k == 0ull ? -1 : (int32_t)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
            *p.ticket = 0u;
        }
    }
}

// output_norm + Q8_1 of the final hidden state in one CTA: y = x / sqrt(mean(x^2) + eps) * w
// (rmsnorm_rows arithmetic; plain Q8_1 when w is null), then quantize_q8_1 per 32-block.
__global__ void __launch_bounds__(1024) lm_norm_quantize_kernel(const float *__restrict__ x,
                                                                const float *__restrict__ w, int k, float eps,
                                                                uint8_t *__restrict__ vy) {
    launch_dependents();
    __shared__ float ws[32];
    __shared__ float yv[kLmMaxK];
    float scale = 1.0f;
    if (w) {
        float ss = 0.0f;
        for (int i = threadIdx.x; i < k; i += blockDim.x) ss = fmaf(x[i], x[i], ss);
#pragma unroll
        for (int m = 16; m > 0; m >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, m);
        if ((threadIdx.x & 31) == 0) ws[threadIdx.x >> 5] = ss;
        __syncthreads();
        float t = (int)(threadIdx.x & 31) < (int)(blockDim.x >> 5) ? ws[threadIdx.x & 31] : 0.0f;
#pragma unroll
        for (int m = 16; m > 0; m >>= 1) t += __shfl_xor_sync(0xffffffffu, t, m);
        scale = rsqrtf(__fdiv_rn(t, (float)k) + eps);
    }
    for (int i = threadIdx.x; i < k; i += blockDim.x) yv[i] = w ? __fmul_rn(__fmul_rn(x[i], scale), w[i]) : x[i];
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int b = warp; b < k / 32; b += blockDim.x >> 5) {
        const float v = yv[32 * b + lane];
        float amax = fabsf(v), sum = v;
#pragma unroll
        for (int m = 16; m > 0; m >>= 1) {
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, m));
            sum += __shfl_xor_sync(0xffffffffu, sum, m);
        }
        const float d = __fdiv_rn(amax, 127.0f);
        const int q = amax == 0.0f ? 0 : (int)roundf(__fdiv_rn(v, d));
        uint8_t *blk = vy + (size_t)b * 36;
        blk[4 + lane] = (uint8_t)q;
        if (lane == 0) {
            *reinterpret_cast<__half *>(blk) = __float2half_rn(d);
            *reinterpret_cast<__half *>(blk + 2) = __float2half_rn(sum);
        }
    }
}

static size_t lm_smem_bytes() {
    return (size_t)kLmSlots * kLmSlotBytes + kLmMaxK / 32 * 36 + sizeof(uint64_t) * (2 * kLmSlots + 1) +
           sizeof(unsigned long long) * kLmConsumers + sizeof(int) * (kLmSlots + 1) + 16;
}

template <int NSB>
static cudaError_t lm_launch_nsb(const LmParams &p, int grid, cudaStream_t s) {
    static std::once_flag once[64];
    int dev = 0;
    cudaGetDevice(&dev);
    std::call_once(once[dev & 63], [] {
        cudaFuncSetAttribute(lm_q6k_kernel<NSB>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)lm_smem_bytes());
    });
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kLmThreads);
    cfg.dynamicSmemBytes = lm_smem_bytes();
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, lm_q6k_kernel<NSB>, p);
}

static int lm_launch(const LmParams &p, cudaStream_t s) {
    if (!p.w || !p.vy || !p.logits || p.rows < 2 || p.k <= 0 || p.k % 256 || p.k > kLmMaxK) return MMRS_ERR_ARG;
    if (((uintptr_t)p.w & 15u) || ((uintptr_t)p.vy & 15u) || (p.token && (!p.best || !p.ticket)))
        return MMRS_ERR_ARG;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int grid = std::max(1, std::min(sms, p.rows / 2));
    if ((p.rows / 2 + grid - 1) / grid * 2 / kLmGroupRows + 2 > kLmMaxGroups) return MMRS_ERR_UNSUPPORTED;
    cudaError_t e;
    switch (p.k / 256) {
        case 4: e = lm_launch_nsb<4>(p, grid, s); break;
        case 8: e = lm_launch_nsb<8>(p, grid, s); break;
        case 12: e = lm_launch_nsb<12>(p, grid, s); break;
        case 16: e = lm_launch_nsb<16>(p, grid, s); break;
        default: return MMRS_ERR_UNSUPPORTED;
    }
    return e == cudaSuccess ? MMRS_OK : MMRS_ERR_LAUNCH;
}

}  // namespace mmrs

using namespace mmrs;

namespace {
struct LmLayout {
    size_t ctl, vy, total;
};
LmLayout lm_layout(const MmrsLmHead *h) {
    LmLayout l{};
    l.ctl = 0;  // [0] status, [1] ticket, [2..3] best (8-byte aligned)
    l.vy = 256;
    l.total = l.vy + ((size_t)h->hidden / 32 * 36 + 255) / 256 * 256;
    return l;
}
}  // namespace

extern "C" void launch_mmvq_gguf_q6_k_f32_plain(const void *vx, const void *vy, void *dst, int ncols_x, int nrows_x,
                                                int stride_col_y, int stride_col_dst, int b_size, void *stream) {
    (void)stride_col_dst;  // one column
    if (b_size != 1) {
        record_error(MMRS_ERR_UNSUPPORTED);
        return;
    }
    if (stride_col_y * 32 < ncols_x) {
        record_error(MMRS_ERR_ARG);
        return;
    }
    LmParams p = {};
    p.w = static_cast<const uint8_t *>(vx);
    p.rows = nrows_x;
    p.k = ncols_x;
    p.vy = static_cast<const uint8_t *>(vy);
    p.logits = static_cast<float *>(dst);
    record_error(lm_launch(p, (cudaStream_t)stream));
}

extern "C" size_t mmrs_lm_head_workspace_bytes(const MmrsLmHead *h) {
    if (!h || h->hidden <= 0 || h->hidden % 256 || h->hidden > kLmMaxK || h->vocab < 2) return 0;
    return lm_layout(h).total;
}

extern "C" int mmrs_lm_head_workspace_status(const void *workspace) {
    if (!workspace) return MMRS_ERR_ARG;
    uint32_t st = 0;
    if (cudaMemcpy(&st, workspace, sizeof(st), cudaMemcpyDeviceToHost) != cudaSuccess) return MMRS_ERR_LAUNCH;
    return (int)st;
}

extern "C" int mmrs_lm_head_forward(const MmrsLmHead *h, const float *x, float *logits, int32_t *token,
                                    void *workspace, size_t workspace_bytes, mmrs_stream_t stream) {
    if (!h || !h->weight || !x || !logits || !workspace) return MMRS_ERR_ARG;
    if (mmrs_lm_head_workspace_bytes(h) == 0) return MMRS_ERR_UNSUPPORTED;
    const LmLayout l = lm_layout(h);
    if (workspace_bytes < l.total || ((uintptr_t)workspace & 255u)) return MMRS_ERR_ARG;
    cudaStream_t s = (cudaStream_t)stream;
    uint8_t *ws = static_cast<uint8_t *>(workspace);
    uint8_t *vy = ws + l.vy;
    lm_norm_quantize_kernel<<<1, 1024, 0, s>>>(x, h->norm_weight, h->hidden, h->eps, vy);
    if (cudaGetLastError() != cudaSuccess) return MMRS_ERR_LAUNCH;
    LmParams p = {};
    p.w = static_cast<const uint8_t *>(h->weight);
    p.rows = h->vocab;
    p.k = h->hidden;
    p.vy = vy;
    p.logits = logits;
    p.token = token;
    uint32_t *ctl = reinterpret_cast<uint32_t *>(ws + l.ctl);
    p.status = ctl;
    p.ticket = ctl + 1;
    p.best = reinterpret_cast<unsigned long long *>(ctl + 2);
    return lm_launch(p, s);
}
