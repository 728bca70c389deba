// Tensor-memory-accelerator (TMA) helpers shared by the prefill GEMM and the decode attention:
// the driver's tensor-map encoder (looked up once through the runtime) and tiled tensor loads.
// No load here uses cluster multicast.
#pragma once

#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"

namespace mmrs {

inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    });
    return fn;
}

// 3-D tiled load into this CTA's shared memory, completion counted on `bar` (x * element size
// must be a multiple of 16 bytes).
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, int x, int y, int z, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}

// Programmatic dependent launch: a kernel launched with the programmatic-serialization attribute
// may start while the previous kernel in the stream still runs; grid_dependency_wait() blocks until
// that kernel has completed and its writes are visible (a no-op without the attribute).
// launch_dependents() lets the next such kernel start early.
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

}  // namespace mmrs
