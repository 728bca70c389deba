// Peer-visible exchange memory for the multi-GPU MoE block (tensor parallel TP=2 and expert
// parallel W=4/8): one region per rank, mapped into the other ranks' address spaces (CUDA IPC
// between processes, or direct peer pointers inside one process).  The ranks' partial hidden
// states are summed over NVLink with peer loads; every wait on a peer flag is bounded.
#pragma once

#include "common.cuh"

namespace mmrs {

constexpr int kMaxRanks = 8;
constexpr int kXchMaxHidden = 8192;   // decode partial rows per buffer
constexpr int kXchMaxCtas = 1024;

// Layout of one rank's exchange region (bytes).  Flags hold the token of the last operation that
// published data (monotonic; readers wait until flag >= token).  Buffers are double buffered by
// token parity: a rank writes buffer (token & 1) only after every peer has published a later
// token than the last reader of that buffer.
//
// The fused decode kernel pushes instead of pulling: each rank stores its partial rows into every
// rank's receive buffer, slot [token & 1][source rank], as 64-bit words {token, f32 bits} (relaxed
// system-scope stores over NVLink), and each rank polls only its own memory until every word it
// needs carries the operation's token.  One NVLink write and no fence: a system-scope release
// costs microseconds, and every poll of a peer's flag is an NVLink round trip.
constexpr size_t kXchStatus = 0;       // u32: MMRS_ERR_TIMEOUT after an expired wait
constexpr size_t kXchAFlags = 8192;    // u32[kXchMaxCtas]: all-reduce kernel, one per CTA
constexpr size_t kXchA2Flags = 12288;  // u32[kXchMaxCtas]: two-shot all-reduce, reduced chunk ready
constexpr size_t kXchDRecv = 16384;    // u64[2][kMaxRanks][kXchMaxHidden]: decode rows received
constexpr size_t kXchAPart = kXchDRecv + 2 * sizeof(unsigned long long) * kMaxRanks * kXchMaxHidden;  // f32[2][cap]

__host__ __device__ inline size_t xch_bytes(size_t ar_capacity) {
    return kXchAPart + 2 * sizeof(float) * ar_capacity;
}

struct PeerView {
    int world, rank;
    uint8_t *mine;
    const uint8_t *peers[kMaxRanks];  // peers[rank] == mine
    size_t ar_capacity;               // floats per all-reduce buffer
};

// Wrap-safe "a >= b" for monotonic tokens.
__device__ __forceinline__ bool token_reached(uint32_t a, uint32_t b) { return (int)(a - b) >= 0; }

// Bounded wait until *flag >= token (system-scope acquire), one memory round trip a poll.  No
// __nanosleep between polls: on B200 a warp woken from it was measured to resume microseconds
// after the requested 32-128 ns.  false on timeout.
__device__ __forceinline__ bool wait_flag_sys(const uint32_t *flag, uint32_t token, uint64_t deadline) {
    uint32_t spins = 0;
    while (!token_reached(ld_acquire_sys(flag), token)) {
        if ((++spins & 63u) == 0 && globaltimer_ns() > deadline) return false;
    }
    return true;
}

// System-scope relaxed loads of peer data (coherent, so never a stale L1 line; unlike volatile
// loads, independent ones stay in flight together).  Issue them after the acquire of the flag
// that published the data and a CTA barrier.
__device__ __forceinline__ float ld_relaxed_sys_f32(const float *p) {
    float v;
    asm volatile("ld.relaxed.sys.global.f32 %0, [%1];" : "=f"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ float4 ld_relaxed_sys_f4(const float4 *p) {
    float4 v;
    asm volatile("ld.relaxed.sys.global.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p));
    return v;
}

// 64-bit relaxed accesses at system scope (the peers' GPUs): a tagged word is written and read
// whole, so a reader that sees the token sees the payload stored with it.
__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long *p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

int peer_all_reduce(const PeerView &g, const float *residual, float *y, size_t count, uint32_t token,
                    uint64_t timeout_ns, cudaStream_t stream);

}  // namespace mmrs
