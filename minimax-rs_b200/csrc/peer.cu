// Peer exchange for the multi-GPU MoE block: allocation and IPC mapping of the exchange regions,
// the multi-rank peer all-reduce (+ residual), and the reference's two-rank peer collectives
// (tp2_peer_all_reduce_f32_cuda1 / tp2_peer_broadcast_f32_cuda1, mmvq_gguf.cu:888-966) with
// bounded waits.
#include <cstring>

#include "peer.cuh"
#include "workspace.cuh"

namespace mmrs {

// Messages of at least this many floats (2 MiB) use the two-shot all-reduce on 4 or more ranks
// (measured on 4 B200s: one round of flags is cheaper below, two-shot ties or beats NCCL above).
constexpr size_t kTwoShotMin = size_t(1) << 19;

// ------------------------------------------------------------------------------------------
// Multi-rank all-reduce: y[i] = (p_0[i] + p_1[i] + ... + p_{W-1}[i]) (+ residual[i]), summed in
// rank order on every rank, so all ranks hold bit-identical results.  p_r is rank r's partial in
// its exchange region, buffer (token & 1).  CTA b owns one contiguous chunk; it publishes its
// own flag (the chunk of the local partial, written by earlier kernels on this stream, is ready),
// waits for the same CTA's flag on every peer, then reads the peers' chunks over NVLink.
// ------------------------------------------------------------------------------------------
struct PeerArParams {
    const float *part[kMaxRanks];
    uint32_t *my_flags, *my_flags2;
    const uint32_t *peer_flags[kMaxRanks], *peer_flags2[kMaxRanks];
    float *my_part;  // this rank's partial (the two-shot kernel writes its reduced chunk there)
    uint32_t *status;
    const float *residual;
    float *y;
    size_t count;
    int world, rank;
    uint32_t token;
    uint64_t timeout_ns;
};

__global__ void __launch_bounds__(256) peer_allreduce_kernel(const PeerArParams p) {
    __shared__ int ok;
    const int b = blockIdx.x;
    const size_t per = ((p.count + gridDim.x - 1) / gridDim.x + 3) / 4 * 4;
    const size_t lo = (size_t)b * per < p.count ? (size_t)b * per : p.count;
    const size_t hi = lo + per < p.count ? lo + per : p.count;
    __syncthreads();
    if (threadIdx.x == 0) {
        const uint64_t deadline = globaltimer_ns() + p.timeout_ns;
        st_release_sys(p.my_flags + b, p.token);
        ok = 1;
        for (int r = 0; r < p.world; ++r) {
            if (r == p.rank) continue;
            if (!wait_flag_sys(p.peer_flags[r] + b, p.token, deadline)) {
                atomicExch(p.status, (uint32_t)MMRS_ERR_TIMEOUT);
                ok = 0;
                break;
            }
        }
    }
    __syncthreads();
    if (!ok) return;
    // float4 body (chunk bounds are multiples of 4), every rank's vector loaded before the sum
    for (size_t i = lo + 4 * threadIdx.x; i + 4 <= hi; i += 4 * blockDim.x) {
        float4 v[kMaxRanks];
#pragma unroll
        for (int r = 0; r < kMaxRanks; ++r)
            if (r < p.world)
                v[r] = r == p.rank ? *reinterpret_cast<const float4 *>(p.part[r] + i)
                                   : ld_relaxed_sys_f4(reinterpret_cast<const float4 *>(p.part[r] + i));
        float4 a = v[0];
#pragma unroll
        for (int r = 1; r < kMaxRanks; ++r)
            if (r < p.world) {
                a.x = a.x + v[r].x;
                a.y = a.y + v[r].y;
                a.z = a.z + v[r].z;
                a.w = a.w + v[r].w;
            }
        if (p.residual) {
            const float4 rr = *reinterpret_cast<const float4 *>(p.residual + i);
            a.x = a.x + rr.x;
            a.y = a.y + rr.y;
            a.z = a.z + rr.z;
            a.w = a.w + rr.w;
        }
        *reinterpret_cast<float4 *>(p.y + i) = a;
    }
    // scalar tail of the last chunk
    for (size_t i = hi - (hi - lo) % 4 + threadIdx.x; i < hi; i += blockDim.x) {
        float v = p.rank == 0 ? p.part[0][i] : ld_relaxed_sys_f32(p.part[0] + i);
        for (int r = 1; r < p.world; ++r) v = v + (r == p.rank ? p.part[r][i] : ld_relaxed_sys_f32(p.part[r] + i));
        if (p.residual) v = v + p.residual[i];
        p.y[i] = v;
    }
}

// ------------------------------------------------------------------------------------------
// Two-shot all-reduce for large messages (W >= 4): chunk r = [r * cs, (r + 1) * cs) is reduced
// by rank r alone (reduce-scatter: the same rank-ordered sum + residual as the one-shot kernel,
// so every rank still ends with bit-identical values), written back over rank r's own partial
// chunk (no other rank reads that chunk of rank r's partial) and published with a second flag;
// then every rank copies the other ranks' reduced chunks (all-gather).  Each rank reads
// 2 (W - 1) / W of the message over NVLink instead of (W - 1) times it.  CTA b owns sub-range b
// of every chunk, so all waits pair CTA b with CTA b of the peers.
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ bool peer_wait_all(const PeerArParams &p, const uint32_t *const *flags, int b,
                                              uint64_t deadline) {
    for (int r = 0; r < p.world; ++r) {
        if (r == p.rank) continue;
        if (!wait_flag_sys(flags[r] + b, p.token, deadline)) {
            atomicExch(p.status, (uint32_t)MMRS_ERR_TIMEOUT);
            return false;
        }
    }
    return true;
}

__global__ void __launch_bounds__(256) peer_allreduce2_kernel(const PeerArParams p, size_t cs, size_t per) {
    __shared__ int ok;
    const int b = blockIdx.x;
    const uint64_t deadline = globaltimer_ns() + p.timeout_ns;
    auto sub = [&](int r, size_t &lo, size_t &hi) {  // sub-range b of chunk r
        const size_t c0 = (size_t)r * cs, c1 = c0 + cs < p.count ? c0 + cs : p.count;
        lo = c0 + (size_t)b * per < c1 ? c0 + (size_t)b * per : c1;
        hi = lo + per < c1 ? lo + per : c1;
    };
    // phase 1: reduce this rank's chunk
    if (threadIdx.x == 0) {
        st_release_sys(p.my_flags + b, p.token);  // the local partial is ready
        ok = peer_wait_all(p, p.peer_flags, b, deadline) ? 1 : 0;
    }
    __syncthreads();
    if (!ok) return;
    size_t lo, hi;
    sub(p.rank, lo, hi);
    for (size_t i = lo + 4 * threadIdx.x; i + 4 <= hi; i += 4 * blockDim.x) {
        float4 v[kMaxRanks];
#pragma unroll
        for (int r = 0; r < kMaxRanks; ++r)
            if (r < p.world)
                v[r] = r == p.rank ? *reinterpret_cast<const float4 *>(p.part[r] + i)
                                   : ld_relaxed_sys_f4(reinterpret_cast<const float4 *>(p.part[r] + i));
        float4 a = v[0];
#pragma unroll
        for (int r = 1; r < kMaxRanks; ++r)
            if (r < p.world) {
                a.x = a.x + v[r].x;
                a.y = a.y + v[r].y;
                a.z = a.z + v[r].z;
                a.w = a.w + v[r].w;
            }
        if (p.residual) {
            const float4 rr = *reinterpret_cast<const float4 *>(p.residual + i);
            a.x = a.x + rr.x;
            a.y = a.y + rr.y;
            a.z = a.z + rr.z;
            a.w = a.w + rr.w;
        }
        *reinterpret_cast<float4 *>(p.my_part + i) = a;
        *reinterpret_cast<float4 *>(p.y + i) = a;
    }
    for (size_t i = hi - (hi - lo) % 4 + threadIdx.x; i < hi; i += blockDim.x) {
        float v = p.rank == 0 ? p.part[0][i] : ld_relaxed_sys_f32(p.part[0] + i);
        for (int r = 1; r < p.world; ++r) v = v + (r == p.rank ? p.part[r][i] : ld_relaxed_sys_f32(p.part[r] + i));
        if (p.residual) v = v + p.residual[i];
        p.my_part[i] = v;
        p.y[i] = v;
    }
    __syncthreads();
    // phase 2: publish the reduced sub-range, gather the peers'
    if (threadIdx.x == 0) {
        st_release_sys(p.my_flags2 + b, p.token);
        ok = peer_wait_all(p, p.peer_flags2, b, deadline) ? 1 : 0;
    }
    __syncthreads();
    if (!ok) return;
    for (int r = 0; r < p.world; ++r) {
        if (r == p.rank) continue;
        sub(r, lo, hi);
        for (size_t i = lo + 4 * threadIdx.x; i + 4 <= hi; i += 4 * blockDim.x)
            *reinterpret_cast<float4 *>(p.y + i) = ld_relaxed_sys_f4(reinterpret_cast<const float4 *>(p.part[r] + i));
        for (size_t i = hi - (hi - lo) % 4 + threadIdx.x; i < hi; i += blockDim.x) p.y[i] = ld_relaxed_sys_f32(p.part[r] + i);
    }
}

int peer_all_reduce(const PeerView &g, const float *residual, float *y, size_t count, uint32_t token,
                    uint64_t timeout_ns, cudaStream_t stream) {
    if (count == 0) return MMRS_OK;
    if (g.world < 1 || g.world > kMaxRanks || g.rank < 0 || g.rank >= g.world || !g.mine || count > g.ar_capacity)
        return MMRS_ERR_ARG;
    // float4 access: 16-byte aligned buffers and an even split of the capacity
    if ((g.ar_capacity & 3u) || ((uintptr_t)y & 15u) || (residual && ((uintptr_t)residual & 15u))) return MMRS_ERR_ARG;
    PeerArParams p = {};
    for (int r = 0; r < g.world; ++r) {
        if (!g.peers[r]) return MMRS_ERR_ARG;
        p.part[r] = reinterpret_cast<const float *>(g.peers[r] + kXchAPart) + (size_t)(token & 1u) * g.ar_capacity;
        p.peer_flags[r] = reinterpret_cast<const uint32_t *>(g.peers[r] + kXchAFlags);
        p.peer_flags2[r] = reinterpret_cast<const uint32_t *>(g.peers[r] + kXchA2Flags);
    }
    p.my_flags = reinterpret_cast<uint32_t *>(g.mine + kXchAFlags);
    p.my_flags2 = reinterpret_cast<uint32_t *>(g.mine + kXchA2Flags);
    p.my_part = reinterpret_cast<float *>(g.mine + kXchAPart) + (size_t)(token & 1u) * g.ar_capacity;
    p.status = reinterpret_cast<uint32_t *>(g.mine + kXchStatus);
    p.residual = residual;
    p.y = y;
    p.count = count;
    p.world = g.world;
    p.rank = g.rank;
    p.token = token;
    p.timeout_ns = timeout_ns;
    if (g.world >= 4 && count >= kTwoShotMin) {
        // chunks of a multiple of 4 floats; ~2K floats of every chunk per CTA
        const size_t cs = ((count + g.world - 1) / g.world + 3) / 4 * 4;
        size_t ctas = (cs + 2047) / 2048;
        if (ctas > 592) ctas = 592;
        const size_t per = ((cs + ctas - 1) / ctas + 3) / 4 * 4;
        peer_allreduce2_kernel<<<(unsigned)ctas, 256, 0, stream>>>(p, cs, per);
        return cudaGetLastError() == cudaSuccess ? MMRS_OK : MMRS_ERR_LAUNCH;
    }
    // one CTA per ~4K floats, at most one wave of the flag array
    size_t ctas = (count + 4095) / 4096;
    if (ctas > (size_t)kXchMaxCtas) ctas = kXchMaxCtas;
    if (ctas > 592) ctas = 592;
    peer_allreduce_kernel<<<(unsigned)ctas, 256, 0, stream>>>(p);
    return cudaGetLastError() == cudaSuccess ? MMRS_OK : MMRS_ERR_LAUNCH;
}

// ------------------------------------------------------------------------------------------
// Reference two-rank collectives.  Signal words (128-byte peer-visible buffers, zeroed once):
// [0] arrival, [1] departure, [2] self epoch counter (epoch == 0 mode); this library adds
// [3] = MMRS_ERR_TIMEOUT when a bounded wait expired.
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ bool tp2_sync(uint32_t *self_signal, uint32_t *peer_signal, int word, uint32_t epoch,
                                         uint64_t deadline) {
    st_release_sys(peer_signal + word, epoch);
    if (!wait_flag_sys(self_signal + word, epoch, deadline)) {
        atomicExch(self_signal + 3, (uint32_t)MMRS_ERR_TIMEOUT);
        return false;
    }
    return true;
}

__global__ void __launch_bounds__(256) tp2_peer_all_reduce_kernel(const float *local, const float *peer,
                                                                  const float *residual, const float *norm_weight,
                                                                  float *output, float *normalized_output,
                                                                  uint32_t *self_signal, uint32_t *peer_signal,
                                                                  uint32_t epoch, int count, float norm_eps,
                                                                  uint64_t timeout_ns) {
    const int tid = threadIdx.x;
    __shared__ uint32_t op_epoch;
    __shared__ int ok;
    __shared__ float sums[256];
    const uint64_t deadline = globaltimer_ns() + timeout_ns;
    if (tid == 0) {
        op_epoch = epoch == 0 ? atomicAdd(self_signal + 2, 1u) + 1u : epoch;
        ok = tp2_sync(self_signal, peer_signal, 0, op_epoch, deadline);
    }
    __syncthreads();
    if (ok) {
        float sq = 0.0f;
        for (int i = tid; i < count; i += blockDim.x) {
            const float reduced = local[i] + ld_relaxed_sys_f32(peer + i);
            const float v = residual ? reduced + residual[i] : reduced;
            output[i] = v;
            sq = fmaf(v, v, sq);
        }
        if (normalized_output) {
            sums[tid] = sq;
            for (int stride = 128; stride > 0; stride >>= 1) {
                __syncthreads();
                if (tid < stride) sums[tid] += sums[tid + stride];
            }
            __syncthreads();
            const float scale = rsqrtf(sums[0] / (float)count + norm_eps);
            for (int i = tid; i < count; i += blockDim.x) normalized_output[i] = output[i] * scale * norm_weight[i];
        }
    }
    __syncthreads();
    if (tid == 0 && ok) tp2_sync(self_signal, peer_signal, 1, op_epoch, deadline);
}

__global__ void __launch_bounds__(256) tp2_peer_broadcast_kernel(const float *source, float *output,
                                                                uint32_t *self_signal, uint32_t *peer_signal,
                                                                uint32_t epoch, int rank, int count,
                                                                uint64_t timeout_ns) {
    const int tid = threadIdx.x;
    __shared__ uint32_t op_epoch;
    __shared__ int ok;
    const uint64_t deadline = globaltimer_ns() + timeout_ns;
    if (tid == 0) {
        op_epoch = epoch == 0 ? atomicAdd(self_signal + 2, 1u) + 1u : epoch;
        ok = tp2_sync(self_signal, peer_signal, 0, op_epoch, deadline);
    }
    __syncthreads();
    if (ok && rank == 1)
        for (int i = tid; i < count; i += blockDim.x) output[i] = source[i];
    __syncthreads();
    if (tid == 0 && ok) tp2_sync(self_signal, peer_signal, 1, op_epoch, deadline);
}

}  // namespace mmrs

using namespace mmrs;

namespace {
constexpr uint64_t kPeerTimeoutNs = 2000000000ull;
int view_of(const MmrsPeerGroup *g, PeerView &v) {
    if (!g || g->world < 1 || g->world > kMaxRanks || g->rank < 0 || g->rank >= g->world || !g->mine)
        return MMRS_ERR_ARG;
    v.world = g->world;
    v.rank = g->rank;
    v.mine = static_cast<uint8_t *>(g->mine);
    for (int r = 0; r < kMaxRanks; ++r) v.peers[r] = static_cast<const uint8_t *>(r < g->world ? g->peers[r] : nullptr);
    v.ar_capacity = g->ar_capacity;
    return MMRS_OK;
}
}  // namespace

extern "C" size_t mmrs_xch_bytes(size_t ar_capacity) { return xch_bytes(ar_capacity); }

extern "C" int mmrs_peer_alloc(size_t bytes, void **ptr) {
    if (!ptr || bytes == 0) return MMRS_ERR_ARG;
    *ptr = nullptr;
    if (cudaMalloc(ptr, bytes) != cudaSuccess) return MMRS_ERR_ALLOC;
    if (cudaMemset(*ptr, 0, bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
        cudaFree(*ptr);
        *ptr = nullptr;
        return MMRS_ERR_LAUNCH;
    }
    return MMRS_OK;
}

extern "C" int mmrs_peer_free(void *ptr) { return cudaFree(ptr) == cudaSuccess ? MMRS_OK : MMRS_ERR_LAUNCH; }

extern "C" int mmrs_ipc_handle(void *ptr, uint8_t *out64) {
    if (!ptr || !out64) return MMRS_ERR_ARG;
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, ptr) != cudaSuccess) return MMRS_ERR_LAUNCH;
    static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
    std::memcpy(out64, &h, sizeof(h));
    return MMRS_OK;
}

extern "C" int mmrs_ipc_open(const uint8_t *handle64, void **ptr) {
    if (!handle64 || !ptr) return MMRS_ERR_ARG;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle64, sizeof(h));
    return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? MMRS_OK : MMRS_ERR_LAUNCH;
}

extern "C" int mmrs_ipc_close(void *ptr) { return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? MMRS_OK : MMRS_ERR_LAUNCH; }

extern "C" int mmrs_peer_enable(int peer_device) {
    int dev = 0, can = 0;
    cudaGetDevice(&dev);
    if (peer_device == dev) return MMRS_OK;
    if (cudaDeviceCanAccessPeer(&can, dev, peer_device) != cudaSuccess || !can) return MMRS_ERR_UNSUPPORTED;
    const cudaError_t e = cudaDeviceEnablePeerAccess(peer_device, 0);
    if (e == cudaErrorPeerAccessAlreadyEnabled) {
        cudaGetLastError();
        return MMRS_OK;
    }
    return e == cudaSuccess ? MMRS_OK : MMRS_ERR_LAUNCH;
}

extern "C" float *mmrs_xch_ar_buffer(const MmrsPeerGroup *g, uint32_t token) {
    if (!g || !g->mine) return nullptr;
    return reinterpret_cast<float *>(static_cast<uint8_t *>(g->mine) + kXchAPart) + (size_t)(token & 1u) * g->ar_capacity;
}

extern "C" int mmrs_peer_all_reduce(const MmrsPeerGroup *g, const float *residual, float *y, size_t count,
                                    uint32_t token, mmrs_stream_t stream) {
    PeerView v;
    int rc = view_of(g, v);
    if (rc != MMRS_OK) return rc;
    if (!y) return MMRS_ERR_ARG;
    return peer_all_reduce(v, residual, y, count, token, kPeerTimeoutNs, (cudaStream_t)stream);
}

extern "C" int mmrs_peer_status(const MmrsPeerGroup *g, mmrs_stream_t stream) {
    if (!g || !g->mine) return MMRS_ERR_ARG;
    uint32_t status = 0;
    cudaStream_t s = (cudaStream_t)stream;
    if (cudaMemcpyAsync(&status, g->mine, sizeof(status), cudaMemcpyDeviceToHost, s) != cudaSuccess)
        return MMRS_ERR_LAUNCH;
    if (cudaStreamSynchronize(s) != cudaSuccess) return MMRS_ERR_LAUNCH;
    if (status) {
        cudaMemsetAsync(g->mine, 0, sizeof(uint32_t), s);
        cudaStreamSynchronize(s);
    }
    return (int)status;
}

extern "C" void launch_tp2_peer_all_reduce_f32(const void *local, const void *peer, const void *residual,
                                               const void *norm_weight, void *output, void *normalized_output,
                                               void *self_signal, void *peer_signal, unsigned int epoch, int count,
                                               float norm_eps, void *stream) {
    if (!local || !peer || !output || !self_signal || !peer_signal || count < 0 ||
        (normalized_output && !norm_weight)) {
        record_error(MMRS_ERR_ARG);
        return;
    }
    tp2_peer_all_reduce_kernel<<<1, 256, 0, (cudaStream_t)stream>>>(
        (const float *)local, (const float *)peer, (const float *)residual, (const float *)norm_weight,
        (float *)output, (float *)normalized_output, (uint32_t *)self_signal, (uint32_t *)peer_signal, epoch, count,
        norm_eps, kPeerTimeoutNs);
    record_error(cudaGetLastError() == cudaSuccess ? MMRS_OK : MMRS_ERR_LAUNCH);
}

extern "C" void launch_tp2_peer_broadcast_f32(const void *source, void *output, void *self_signal, void *peer_signal,
                                              unsigned int epoch, int rank, int count, void *stream) {
    if (!output || !self_signal || !peer_signal || count < 0 || (rank == 1 && !source)) {
        record_error(MMRS_ERR_ARG);
        return;
    }
    tp2_peer_broadcast_kernel<<<1, 256, 0, (cudaStream_t)stream>>>((const float *)source, (float *)output,
                                                                   (uint32_t *)self_signal, (uint32_t *)peer_signal,
                                                                   epoch, rank, count, kPeerTimeoutNs);
    record_error(cudaGetLastError() == cudaSuccess ? MMRS_OK : MMRS_ERR_LAUNCH);
}
