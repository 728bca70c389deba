// Single-token MoE block that allocates nothing.
//
// Some callers cannot allocate device memory at the moment they run the MoE block: a host engine
// whose device memory is entirely pre-reserved by its own allocator, or a call site shaped like
// the reference's FFI that hands over only tensor pointers and has no workspace to pass (the
// reference's own launchers fall back to cudaMallocAsync, which needs a stream-ordered pool that
// may be disabled or exhausted).  For them this file keeps the scratch of the fused decode kernel
// in a fixed, file-scope device array: every GPU that loads the library holds it until exit.
//
// Limits: num_experts <= 256, inter <= 1536, hidden <= 3072 (the scratch layout of the fused
// decode kernel for those sizes fits kStaticScratchBytes).  Larger problems are rejected with
// MMRS_ERR_SCRATCH_LIMIT before anything is launched.
//
// The scratch is shared by every call on a device and keeps the last call's contents.  Each call
// starts at zero and is never cleared between calls: its launch tags keep counting, so the
// tagged words a call hands between CTAs never match a stale word of an earlier call
// (mmrs_moe_static_status clears it after a call that failed).  Calls that overlap
// on the GPU (different streams or host threads without ordering) race on the scratch.
//
// The first call on a device resolves the device address of the array (cudaGetSymbolAddress, with
// that device current) and caches it; make that first call before any stream capture.  The cached
// address belongs to the device's current context: do not use these entry points across a
// cudaDeviceReset (or any other teardown of the primary context) in the same process.
//
// A bounded device-side wait that expires leaves MMRS_ERR_TIMEOUT in the array's status word and
// y unwritten; mmrs_moe_static_status() reads and clears that word (the next call clears it too,
// so read it before the next call).
#include <mutex>

#include "common.cuh"
#include "decode.cuh"
#include "workspace.cuh"

namespace mmrs {

constexpr int kStaticMaxExperts = 256;
constexpr int kStaticMaxInter = 1536;
constexpr int kStaticMaxHidden = 3072;
constexpr size_t kStaticScratchBytes = 128 * 1024;

static __device__ __align__(256) uint8_t g_decode_scratch[kStaticScratchBytes];

static std::mutex g_scratch_mu;
static void *g_scratch_addr[64];

// Device address of g_decode_scratch on the current device, cached per device and checked on
// every call: after a device reset the context (and the array's address) is new, so a cached
// address that no longer resolves to device memory of this context is looked up again (the array
// itself is zero again then, as its launch tags require).
static int scratch_address(void **out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return MMRS_ERR_LAUNCH;
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (g_scratch_addr[dev]) {
        cudaPointerAttributes a = {};
        if (cudaPointerGetAttributes(&a, g_scratch_addr[dev]) != cudaSuccess || a.type != cudaMemoryTypeDevice ||
            a.device != dev) {
            cudaGetLastError();  // clear the lookup's error state
            g_scratch_addr[dev] = nullptr;
        }
    }
    if (!g_scratch_addr[dev]) {
        void *ptr = nullptr;
        if (cudaGetSymbolAddress(&ptr, g_decode_scratch) != cudaSuccess || !ptr) return MMRS_ERR_LAUNCH;
        g_scratch_addr[dev] = ptr;
    }
    *out = g_scratch_addr[dev];
    return MMRS_OK;
}

}  // namespace mmrs

using namespace mmrs;

extern "C" int mmrs_moe_block_decode_static(const MmrsMoeWeights *w, const float *x, const float *residual, float *y,
                                            uint32_t *topk_ids, float *topk_weights, mmrs_stream_t stream) {
    int rc = validate_weights(w);
    if (rc != MMRS_OK) return rc;
    if (!x || !y || (reinterpret_cast<uintptr_t>(x) & 15u)) return MMRS_ERR_ARG;
    if (w->num_experts > kStaticMaxExperts || w->inter > kStaticMaxInter || w->hidden > kStaticMaxHidden)
        return MMRS_ERR_SCRATCH_LIMIT;
    const WsLayout l = ws_layout(w->num_experts, w->inter, 1);
    if (l.total > kStaticScratchBytes) return MMRS_ERR_SCRATCH_LIMIT;
    void *base = nullptr;
    rc = scratch_address(&base);
    if (rc != MMRS_OK) return rc;

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
    ws_bind(p, (uint8_t *)base, l);
    p.trace = nullptr;
    p.E = w->num_experts;
    p.H = w->hidden;
    p.I = w->inter;
    p.gu_type = w->gate_up_type;
    p.dn_type = w->down_type;
    p.timeout_ns = 2000000000ull;
    int dev = 0, sms = 0, smem = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    rc = decode_configure(p, sms, smem);
    if (rc != MMRS_OK) return rc;
    if ((size_t)p.grid > (size_t)kDecodeMaxCtas) return MMRS_ERR_UNSUPPORTED;
    // the scratch starts at zero (a device array) and its launch tags keep counting from call to
    // call: nothing is cleared here (mmrs_moe_static_status clears it after a failed call)
    return decode_launch(p, (cudaStream_t)stream);
}

extern "C" int mmrs_moe_static_status(mmrs_stream_t stream) {
    void *base = nullptr;
    int rc = scratch_address(&base);
    if (rc != MMRS_OK) return rc;
    cudaStream_t s = (cudaStream_t)stream;
    uint32_t status = 0;
    // the status word is the first field of the control block at the start of the array
    if (cudaMemcpyFromSymbolAsync(&status, g_decode_scratch, sizeof(status), 0, cudaMemcpyDeviceToHost, s) !=
        cudaSuccess)
        return MMRS_ERR_LAUNCH;
    if (cudaStreamSynchronize(s) != cudaSuccess) return MMRS_ERR_LAUNCH;
    if (status != 0) {
        // the whole scratch: control block, trace and tagged records
        if (cudaMemsetAsync(base, 0, kStaticScratchBytes, s) != cudaSuccess || cudaStreamSynchronize(s) != cudaSuccess)
            return MMRS_ERR_LAUNCH;
    }
    return (int)status;
}
