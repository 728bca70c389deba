// Measured dense int8 tensor-core throughput of this GPU (the denominator of the prefill GEMM's
// tensor fraction): every SM issues back-to-back tcgen05.mma.kind::i8 of the largest single-CTA
// shape (M = 128, N = 256, K = 32) from operands resident in shared memory into one TMEM
// accumulator, so nothing but the tensor pipe is timed.  The operand bytes are zero: the MMA
// timing does not depend on the values.
#include "../../include/minimax_bench.h"
#include "common.cuh"
#include "umma.cuh"

namespace mmrs {
namespace {

constexpr int kPkM = 128, kPkN = 256, kPkKBytes = 256;  // one 256-byte K chunk: 8 MMAs of K = 32
constexpr int kPkTmemCols = 256;
constexpr int kPkSmem = (kPkM + kPkN) * kPkKBytes + 128;

__global__ void __launch_bounds__(128, 1) int8_peak_kernel(int chunks, uint32_t *status, uint64_t timeout_ns) {
    extern __shared__ __align__(128) uint8_t raw[];
    __shared__ uint32_t tmem_base;
    __shared__ __align__(8) uint64_t done;
    const int tid = threadIdx.x, warp = tid >> 5;
    uint8_t *a = raw, *b = raw + kPkM * kPkKBytes;
    for (int i = tid; i < (kPkM + kPkN) * kPkKBytes / 16; i += blockDim.x) reinterpret_cast<uint4 *>(raw)[i] = make_uint4(0, 0, 0, 0);
    if (tid == 0) {
        mbar_init(&done, 1);
        fence_mbar_init();
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base)),
                     "r"(kPkTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    // the operands were written by generic stores; the tensor pipe reads them through the async proxy
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base;
    if (tid == 0) {
        // canonical no-swizzle K-major layout: 8-row groups of sixteen 8 x 16-byte core matrices
        // (2048 B a group), K-adjacent core matrices 128 B apart; MMA j reads K bytes 32j..32j+31
        const uint32_t abase = smem_u32(a), bbase = smem_u32(b), idesc = umma_idesc_i8(kPkM, kPkN);
        for (int c = 0; c < chunks; ++c) {
#pragma unroll
            for (int j = 0; j < kPkKBytes / 32; ++j)
                tc_mma_i8(tmem, umma_smem_desc(abase + j * 256, 128, 2048), umma_smem_desc(bbase + j * 256, 128, 2048),
                          idesc, (c | j) ? 1u : 0u);
        }
        tc_commit(&done);
        if (!mbar_wait_bounded(&done, 0u, globaltimer_ns() + timeout_ns)) atomicExch(status, (uint32_t)MMRS_ERR_TIMEOUT);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kPkTmemCols));
    }
}

}  // namespace
}  // namespace mmrs

using namespace mmrs;

extern "C" int mmrs_int8_tensor_peak(int chunks, int reps, double *tops, mmrs_stream_t stream) {
    if (!tops || chunks <= 0 || reps <= 0) return MMRS_ERR_ARG;
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return MMRS_ERR_LAUNCH;
    if (cudaFuncSetAttribute(int8_peak_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kPkSmem) != cudaSuccess)
        return MMRS_ERR_LAUNCH;
    cudaStream_t s = (cudaStream_t)stream;
    uint32_t *status = nullptr;
    if (cudaMallocAsync((void **)&status, sizeof(uint32_t), s) != cudaSuccess) return MMRS_ERR_ALLOC;
    cudaMemsetAsync(status, 0, sizeof(uint32_t), s);
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    int8_peak_kernel<<<sms, 128, kPkSmem, s>>>(chunks, status, 2000000000ull);  // warm-up
    float best_ms = 0.f;
    for (int r = 0; r < reps; ++r) {
        cudaEventRecord(e0, s);
        int8_peak_kernel<<<sms, 128, kPkSmem, s>>>(chunks, status, 2000000000ull);
        cudaEventRecord(e1, s);
        cudaEventSynchronize(e1);
        float ms = 0.f;
        cudaEventElapsedTime(&ms, e0, e1);
        if (r == 0 || ms < best_ms) best_ms = ms;
    }
    uint32_t st = 0;
    cudaMemcpyAsync(&st, status, sizeof(st), cudaMemcpyDeviceToHost, s);
    cudaStreamSynchronize(s);
    cudaFreeAsync(status, s);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    if (cudaGetLastError() != cudaSuccess) return MMRS_ERR_LAUNCH;
    if (st != 0) return (int)st;
    const double ops = 2.0 * kPkM * kPkN * 32 * (kPkKBytes / 32) * (double)chunks * sms;
    *tops = ops / (best_ms * 1e-3) / 1e12;
    return MMRS_OK;
}
