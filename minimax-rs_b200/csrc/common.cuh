// Shared device helpers for the MiniMax MoE hot path on B200 (sm_100a).
//
// GGUF k-quant block layouts (byte-compatible with the reference's vendored Candle kernels,
// candle-kernels/src/moe/gguf.cuh:341-406):
//   Q4_K  144 B per 256 weights: half2 dm | 12 B packed 6-bit scales+mins | 128 B nibbles
//   Q5_K  176 B per 256 weights: half2 dm | 12 B scales+mins | 32 B high bits | 128 B nibbles
//   Q8_1   36 B per  32 values : half2 (d, sum) | 32 x int8
// Element order inside a super-block (quantized.cu:943-1004): element 64j+l is the low nibble of
// qs[32j+l] (sub-block 2j), element 64j+32+l the high nibble (sub-block 2j+1); Q5_K adds 16 when
// bit 2j (resp. 2j+1) of qh[l] is set.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/minimax_moe.h"

namespace mmrs {

constexpr int QK_K = 256;
constexpr int Q4K_BYTES = 144;
constexpr int Q5K_BYTES = 176;
constexpr int Q81_BYTES = 36;

__host__ __device__ inline int kq_block_bytes(int t) { return t == MMRS_Q5K ? Q5K_BYTES : Q4K_BYTES; }
__host__ __device__ inline size_t kq_row_bytes(int t, int k) { return (size_t)(k / QK_K) * kq_block_bytes(t); }
__host__ __device__ inline int pad_to(int v, int p) { return (v + p - 1) / p * p; }

// Exact integer -> float conversions that stay off the conversion pipe (a quarter-rate unit):
// the integer is placed in the mantissa of a power of two and that power is subtracted.
// small_uint_to_float: 0 <= v < 2^23.  int22_to_float: -2^22 <= v < 2^22.
__device__ __forceinline__ float small_uint_to_float(uint32_t v) {
    return __uint_as_float(0x4B000000u | v) - 8388608.0f;
}
__device__ __forceinline__ float int22_to_float(int v) {
    return __int_as_float(0x4B400000 + v) - 12582912.0f;
}

__device__ __forceinline__ float half_bits_to_float(uint32_t bits16) {
    return __half2float(__ushort_as_half((unsigned short)(bits16 & 0xffffu)));
}

// ------------------------------------------------------------------------------------------
// Warp helpers
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum_butterfly(float v) {
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
    return v;
}
__device__ __forceinline__ float warp_max_butterfly(float v) {
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, m));
    return v;
}

// ------------------------------------------------------------------------------------------
// Time (ns) for bounded waits
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ------------------------------------------------------------------------------------------
// mbarrier + bulk async copy (TMA, non-tensor) wrappers
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile(
        "{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
            smem_u32(bar)),
        "r"(bytes)
        : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Non-blocking test of a phase (mbarrier.try_wait without a hint costs ~0.2 us even on a phase
// that has already completed).
__device__ __forceinline__ bool mbar_test_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait: returns false when the deadline (globaltimer ns) passes.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, uint64_t deadline) {
    if (mbar_test_wait(bar, parity)) return true;
    uint32_t spins = 0;
    while (!mbar_try_wait(bar, parity)) {
        if ((++spins & 1023u) == 0 && globaltimer_ns() > deadline) return false;
    }
    return true;
}
// Bounded wait that lets the waiting warp sleep in hardware (try_wait with a suspend-time hint)
// instead of spinning on issue slots the working warps need.
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t *bar, uint32_t parity, uint64_t deadline) {
    if (mbar_test_wait(bar, parity)) return true;
    for (;;) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(smem_u32(bar)), "r"(parity), "r"(20000u)
            : "memory");
        if (ok) return true;
        if (globaltimer_ns() > deadline) return false;
    }
}

// Ring slot hand-over for consumers that may run more than one fill ahead of a slot: the
// producer stores the index of the fill it is about to issue into ticket[slot]; a consumer waits
// for its fill's index there before the parity wait, which could otherwise match the completed
// phase of an older fill with the same parity.  Bounded by the deadline.
__device__ __forceinline__ bool ring_wait(uint64_t *full, const int *ticket, int slot, int fill, int slots,
                                          uint64_t deadline) {
    uint32_t spins = 0;
    while (*reinterpret_cast<const volatile int *>(&ticket[slot]) != fill) {  // no __nanosleep: see grid_sync
        if ((++spins & 1023u) == 0 && globaltimer_ns() > deadline) return false;
    }
    return mbar_wait_sleep(&full[slot], (uint32_t)(fill / slots) & 1u, deadline);
}

// 1-D bulk copy global -> shared, completion counted on an mbarrier (bytes % 16 == 0,
// both addresses 16-byte aligned).
__device__ __forceinline__ void bulk_g2s(void *smem_dst, const void *gmem_src, uint32_t bytes,
                                         uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(smem_dst)),
        "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void prefetch_l2_bulk(const void *gmem_src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(gmem_src), "r"(bytes) : "memory");
}

// ------------------------------------------------------------------------------------------
// Global acquire / release helpers for the software grid barrier and peer flags.
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_gpu(uint32_t *p, uint32_t v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_gpu_u64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint32_t ld_relaxed_gpu(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_relaxed_gpu_add(uint32_t *p, uint32_t v) {
    asm volatile("red.relaxed.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_relaxed_gpu_u64(unsigned long long *p, unsigned long long v) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// Publishes a 64-bit word for other CTAs with an atomic exchange performed at L2 (the old value
// discarded); the routing scores use it (measured ~0.3 us earlier at the polling CTAs than a
// relaxed store).
__device__ __forceinline__ void publish_gpu_u64(unsigned long long *p, unsigned long long v) {
    unsigned long long old;
    asm volatile("atom.relaxed.gpu.global.exch.b64 %0, [%1], %2;" : "=l"(old) : "l"(p), "l"(v) : "memory");
    (void)old;
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Greedy-choice key of a float (-0 == +0; NaN below every number) and the lowest index among
// equal values: larger key = larger value, then smaller index.  The maximum over a vector is
// its argmax (candle's argmax: the first index of the largest value).
__device__ __forceinline__ unsigned long long lm_key(float v, int idx) {
    v = v + 0.0f;  // -0 -> +0
    uint32_t u = __float_as_uint(v);
    uint32_t o = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    if (v != v) o = 0u;
    return ((unsigned long long)o << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)idx);
}

// Named barrier `id` over `nthreads` threads of the CTA.
__device__ __forceinline__ void named_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}
__device__ __forceinline__ void named_arrive(int id, int nthreads) {
    asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Control block at the start of every workspace: a status word, a grid-arrival counter and one
// epoch word per CTA.  Grid barrier k of a launch: every CTA adds 1 to `count` (fire-and-forget
// red.release) and waits until count >= G * (epoch + k), where epoch is the value of its own
// epoch word at launch start (2 per completed launch: every launch passes exactly two barriers).
// The counter is never reset; comparisons are wrap-safe.
constexpr int kMaxGridCtas = 960;
struct GridFlags {
    uint32_t status;  // MMRS_OK, or MMRS_ERR_TIMEOUT once any wait expired
    uint32_t pad0[31];
    uint32_t count;  // own 128-byte line
    uint32_t pad1[31];
    uint32_t epoch[kMaxGridCtas];
};
constexpr size_t kControlBytes = sizeof(GridFlags);

// Call with `nthreads` threads of the CTA that use named barrier `bar_id`.  Returns false (and
// records MMRS_ERR_TIMEOUT) when the deadline passes.  *s_ok must be 1 on first use.
__device__ inline bool grid_sync(GridFlags *gf, uint32_t target, uint64_t deadline, volatile int *s_ok, int bar_id,
                                 int nthreads) {
    named_sync(bar_id, nthreads);
    if (threadIdx.x == 0 && *s_ok) {
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(&gf->count) : "memory");
        uint32_t spins = 0;
        // one L2 round trip a poll; no __nanosleep between polls (a warp woken from it was
        // measured to resume microseconds after the requested time)
        while ((int)(ld_acquire_gpu(&gf->count) - target) < 0) {
            if ((++spins & 63u) == 0 && globaltimer_ns() > deadline) {
                atomicExch(&gf->status, (uint32_t)MMRS_ERR_TIMEOUT);
                *s_ok = 0;
                break;
            }
        }
    }
    named_sync(bar_id, nthreads);
    return *s_ok != 0;
}

}  // namespace mmrs
