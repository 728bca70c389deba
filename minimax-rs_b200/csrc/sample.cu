// Token sampling over a decode step's logits on B200 (sm_100a): greedy, top-k, top-p (nucleus),
// temperature, and one token's log-probability.
//
// Reference (minimax-rs, src/sampling.rs): TokenSampler::sample (:84-150) copies the whole
// vocabulary to the host for stochastic decoding, partially selects the top_k largest, sorts
// them for top-p, and walks exp((l - max) / T) weights against one uniform draw; token_logprob
// (:60-75) is a log-softmax read at one id.  Here one cooperative launch (one CTA per SM, 512
// threads) does the work where the logits are, reading them once (0.8 MB at 200064 ids, from L2
// right after the LM head wrote them):
//   phase 0  each CTA loads its contiguous slice as 52-bit keys in shared memory: the float's
//            total-order bits << 20 | (2^20 - 1 - id), so a larger key is a larger logit, then a
//            smaller id (the reference's compare_candidates); it notes non-finite values and its
//            largest key, and histograms the keys' top 13 bits;
//   rounds   radix selection of the k-th largest key, 13 bits a round (at most 4 rounds, one
//            grid barrier each): every CTA adds its shared-memory histogram into a global one, and
//            after the barrier every CTA scans the same global histogram, so all agree on the next
//            digit without another exchange.  When a list of at most 1024 keys will do (top-p, or
//            top_k <= 1024), selection stops at the first round whose digit leaves at most 1024
//            keys at or above it — usually the first round — and the list's owner sorts them;
//   list     CTAs append those keys to a global list; the last CTA to finish sorts it (bitonic,
//            shared memory), keeps the top_k, cuts them where the cumulative weight reaches top_p
//            of the total (or orders them by id when there is no top-p cut) and draws;
//   walk     top_k > 1024 (or none) without top-p: the exact k-th key is selected, every CTA sums
//            its candidates' weights (ids ascending), one more barrier lets every CTA form the
//            same prefix over CTAs, and the CTA whose range holds u * total walks its slice.
// Weights and sums are double, as the reference's; the token-log-probability call is one barrier
// and a sum of exp(l - max).  The grid barrier is the bounded software
// barrier of common.cuh (epoch words in the workspace); nothing else waits.
#include <cuda_runtime.h>
#include <math.h>
#include <stddef.h>

#include "../../include/minimax_sample.h"
#include <mutex>

#include "common.cuh"

namespace mmrs {
namespace {

constexpr int kSpThreads = 512;
constexpr int kSpWarps = kSpThreads / 32;
constexpr int kSpIdBits = 20;
constexpr uint32_t kSpIdMask = (1u << kSpIdBits) - 1u;
constexpr int kSpDigitBits = 13;
constexpr int kSpBins = 1 << kSpDigitBits;
constexpr int kSpRounds = 4;  // 4 x 13 = 52 key bits
constexpr int kSpBinsPerThread = kSpBins / kSpThreads;
constexpr int kSpMaxSlice = 8192;  // keys a CTA holds in shared memory
constexpr int kSpMaxSorted = MMRS_SAMPLE_MAX_SORTED;
constexpr uint64_t kSpTimeoutNs = 2000000000ull;
static_assert(kSpMaxSorted == 2 * kSpThreads, "the sorted list is two entries per thread");
static_assert(kSpBins % kSpThreads == 0, "whole bins per thread");

// kList: the candidates end in one list of at most 1024 keys that the last CTA finishes (top-p, or
// top_k <= 1024); kIdWalk: top_k > 1024 (or none) without top-p, walked across the CTAs by id.
enum SpMode : int { kGreedy = 0, kList = 1, kIdWalk = 2, kLogprob = 3 };

// Flags in SpMisc::flags (cleared by the last CTA of every call).
constexpr uint32_t kFlagNonfinite = 1u;
constexpr uint32_t kFlagInternal = 2u;  // a selection round found no digit (cannot happen)

struct SpMisc {
    unsigned long long best;  // greedy: packed maximum (zero between calls)
    uint32_t ticket;          // CTAs done (zero between calls)
    uint32_t ncand;           // entries appended to the sorted list (zero between calls)
    uint32_t flags;           // kFlag* seen in this call (zero between calls)
    uint32_t result;          // outcome of the last completed call
};

struct SpLayout {
    size_t ctl, misc, cta_max, partial, hist, cand, total;
};

SpLayout sp_layout() {
    auto up = [](size_t v) { return (v + 255) / 256 * 256; };
    SpLayout l{};
    l.ctl = 0;
    l.misc = up(kControlBytes);
    l.cta_max = l.misc + 256;
    l.partial = l.cta_max + up(sizeof(unsigned long long) * kMaxGridCtas);
    l.hist = l.partial + up(sizeof(double) * kMaxGridCtas);
    l.cand = l.hist + sizeof(uint32_t) * kSpRounds * 2 * kSpBins;
    l.total = l.cand + sizeof(unsigned long long) * kSpMaxSorted;
    return l;
}

struct SpParams {
    const float *logits;
    int V, chunk, mode;
    int kA, kB;           // ranks to select (0: no selection, every key qualifies)
    int list_n;           // kList: entries kept (min(top_k, 1024))
    int sorted;           // kList: top-p cut (candidates in sorted order), else ascending id
    int s_from_partials;  // top-p total over a candidate set larger than the list
    int token_id;         // kLogprob
    double top_p, temperature, u;
    int32_t *token;
    float *out;
    GridFlags *ctl;
    SpMisc *misc;
    unsigned long long *cta_max;
    double *partial;
    uint32_t *hist;  // [round][search][bin]
    unsigned long long *cand;
};

// Total order of f32 bit patterns (f32::total_cmp: -0 below +0).
__device__ __forceinline__ uint32_t sp_order(float v) {
    const uint32_t u = __float_as_uint(v);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ double sp_logit(unsigned long long key) {
    const uint32_t o = (uint32_t)(key >> kSpIdBits);
    return (double)__uint_as_float((o & 0x80000000u) ? (o & 0x7FFFFFFFu) : ~o);
}
__device__ __forceinline__ int sp_id(unsigned long long key) {
    return (int)(kSpIdMask - (uint32_t)(key & kSpIdMask));
}

template <typename T>
__device__ __forceinline__ T warp_incl_scan(T v, int lane) {
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const T n = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += n;
    }
    return v;
}

// Exclusive prefix of v over the CTA's threads in thread order, and the total (the same
// summation tree on every call).  All threads call it; `sw` holds kSpWarps + 1 values.
template <typename T>
__device__ T block_excl_scan(T v, T *sw, T &total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const T inc = warp_incl_scan(v, lane);
    __syncthreads();
    if (lane == 31) sw[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        const T w = lane < kSpWarps ? sw[lane] : T(0);
        const T wi = warp_incl_scan(w, lane);
        const T we = __shfl_up_sync(0xffffffffu, wi, 1);
        if (lane < kSpWarps) sw[lane] = lane ? we : T(0);
        if (lane == kSpWarps - 1) sw[kSpWarps] = wi;
    }
    __syncthreads();
    T ex = __shfl_up_sync(0xffffffffu, inc, 1);
    if (lane == 0) ex = T(0);
    total = sw[kSpWarps];
    return sw[warp] + ex;
}

__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long n = __shfl_xor_sync(0xffffffffu, v, o);
        v = n > v ? n : v;
    }
    return v;
}

struct SpShared {
    double sw_d[kSpWarps + 1];
    uint32_t sw_u[kSpWarps + 1];
    unsigned long long max_key, gmax_key;
    int ok;
    uint32_t epoch;
    uint32_t flags;              // the call's flags, as read after the first barrier
    int digit, above, in_bin;    // sp_scan's answer
    int first, last;             // smallest / largest index a search found
    int is_last;                 // this CTA finished last
    int status;
    int last_nz;                 // last CTA with a positive partial sum
};

// Histogram of round r for the active searches over the CTA's keys, added into the global one.
__device__ void sp_histogram(const SpParams &p, const unsigned long long *keys, int n, uint32_t *sh, int r,
                             const unsigned long long *prefix, const bool *act) {
    const int tid = threadIdx.x;
    const int shift = (kSpRounds - 1 - r) * kSpDigitBits;
    const int b0 = act[0] ? 0 : kSpBins, b1 = act[1] ? 2 * kSpBins : kSpBins;
    for (int b = b0 + tid; b < b1; b += kSpThreads) sh[b] = 0u;
    __syncthreads();
    for (int i = tid; i < n; i += kSpThreads) {
        const unsigned long long key = keys[i];
#pragma unroll
        for (int s = 0; s < 2; ++s)
            if (act[s] && (key >> (shift + kSpDigitBits)) == prefix[s])
                atomicAdd(&sh[s * kSpBins + (int)((key >> shift) & (kSpBins - 1))], 1u);
    }
    __syncthreads();
    uint32_t *gh = p.hist + (size_t)r * 2 * kSpBins;
    for (int b = b0 + tid; b < b1; b += kSpThreads)
        if (sh[b]) atomicAdd(&gh[b], sh[b]);
}

// Digit of round r for search `srch`: the largest d with (count in bins above d) < need.  Returns d
// (-1 when the histogram holds fewer than `need` keys), the count above it and the count in it.
__device__ int sp_scan(const SpParams &p, SpShared &s, int r, int srch, uint32_t need, uint32_t *above,
                       uint32_t *in_bin) {
    const int tid = threadIdx.x;
    const uint32_t *gh = p.hist + ((size_t)r * 2 + srch) * kSpBins;
    const int top = kSpBins - 1 - tid * kSpBinsPerThread;  // this thread: digits top, top-1, ...
    static_assert(kSpBinsPerThread == 16, "four 16-byte loads a thread");
    uint4 v[4];
    const uint4 *src = reinterpret_cast<const uint4 *>(gh + top - (kSpBinsPerThread - 1));
#pragma unroll
    for (int q = 0; q < 4; ++q) v[q] = __ldcg(src + q);
    const uint32_t *flat = reinterpret_cast<const uint32_t *>(v);
    uint32_t c[kSpBinsPerThread];
    uint32_t sum = 0;
#pragma unroll
    for (int j = 0; j < kSpBinsPerThread; ++j) {
        c[j] = flat[kSpBinsPerThread - 1 - j];
        sum += c[j];
    }
    if (tid == 0) s.digit = -1;
    uint32_t tot;
    const uint32_t ex = block_excl_scan(sum, s.sw_u, tot);  // (its barriers order the store above)
    if (ex < need && need <= ex + sum) {
        uint32_t run = ex;
#pragma unroll
        for (int j = 0; j < kSpBinsPerThread; ++j) {
            if (run + c[j] >= need) {
                s.digit = top - j;
                s.above = (int)run;
                s.in_bin = (int)c[j];
                break;
            }
            run += c[j];
        }
    }
    __syncthreads();
    const int d = s.digit;
    *above = (uint32_t)s.above;
    *in_bin = (uint32_t)s.in_bin;
    __syncthreads();  // (the next scan resets s.digit)
    return d;
}

__device__ bool sp_grid_sync(const SpParams &p, SpShared &s, int &nsync, uint64_t deadline) {
    ++nsync;
    return grid_sync(p.ctl, (uint32_t)gridDim.x * (s.epoch + (uint32_t)nsync), deadline, &s.ok, 1, kSpThreads);
}

// Bitonic sort of n2 (a power of two, <= 1024) keys into descending order.
__device__ void sp_sort_desc(unsigned long long *k, int n2) {
    const int tid = threadIdx.x;
    for (int size = 2; size <= n2; size <<= 1) {
        for (int j = size >> 1; j > 0; j >>= 1) {
            if (tid < n2 / 2) {
                const int i = 2 * j * (tid / j) + (tid % j), l = i + j;
                const unsigned long long a = k[i], b = k[l];
                const bool desc = (i & size) == 0;
                if (desc ? (a < b) : (a > b)) {
                    k[i] = b;
                    k[l] = a;
                }
            }
            __syncthreads();
        }
    }
}

// Sort of at most 64 keys into descending order by warp 0 in registers (lane l holds entries l
// and l + 32); the other warps wait at the closing barrier.
__device__ void sp_warp_sort64_desc(unsigned long long *k, int n) {
    const int lane = threadIdx.x & 31;
    if (threadIdx.x < 32) {
        unsigned long long x[2] = {lane < n ? k[lane] : 0ull, lane + 32 < n ? k[lane + 32] : 0ull};
#pragma unroll
        for (int size = 2; size <= 64; size <<= 1) {
#pragma unroll
            for (int j = size >> 1; j > 0; j >>= 1) {
                if (j == 32) {
                    if (x[0] < x[1]) {  // entries l and l + 32 of the one block of 64: descending
                        const unsigned long long t = x[0];
                        x[0] = x[1];
                        x[1] = t;
                    }
                } else {
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int i = lane + 32 * h;
                        const unsigned long long y = __shfl_xor_sync(0xffffffffu, x[h], j);
                        const bool lower = (i & j) == 0, desc = (i & size) == 0;
                        const unsigned long long hi = x[h] > y ? x[h] : y, lo = x[h] > y ? y : x[h];
                        x[h] = (desc == lower) ? hi : lo;
                    }
                }
            }
        }
        k[lane] = x[0];
        k[lane + 32] = x[1];
    }
    __syncthreads();
}

// Inclusive cumulative weights of a list of 1024 (two entries per thread: 2t, 2t + 1).
__device__ void sp_cumulate(const double *w, double *cum, SpShared &s, double *total) {
    const int tid = threadIdx.x;
    const double a = w[2 * tid], b = w[2 * tid + 1];
    double tot;
    const double ex = block_excl_scan(a + b, s.sw_d, tot);
    cum[2 * tid] = ex + a;
    cum[2 * tid + 1] = (ex + a) + b;
    *total = tot;
    __syncthreads();
}

// The CTAs' partial sums, loaded in parallel, and their running sum in CTA order (one thread, the
// same additions in every CTA): pre[c] = the partials before CTA c, pre[G] = the total.  Also the
// last CTA with a positive partial.
__device__ void sp_cta_prefix(const SpParams &p, SpShared &s, double *vals, double *pre) {
    const int tid = threadIdx.x, G = (int)gridDim.x;
    for (int c = tid; c < G; c += kSpThreads) vals[c] = __ldcg(p.partial + c);
    __syncthreads();
    if (tid == 0) {
        double run = 0.0;
        int last_nz = -1;
        for (int c = 0; c < G; ++c) {
            pre[c] = run;
            if (vals[c] > 0.0) last_nz = c;
            run += vals[c];
        }
        pre[G] = run;
        s.last_nz = last_nz;
    }
    __syncthreads();
}

// Scratch of the last CTA (the histogram space): sorted keys | weights | cumulative weights |
// logits | ids | CTA partials | their prefix.
struct SpScratch {
    unsigned long long *sk;
    double *w, *cum, *lg;
    int *ids;
    double *vals, *pre;
    __device__ explicit SpScratch(unsigned char *b)
        : sk(reinterpret_cast<unsigned long long *>(b)),
          w(reinterpret_cast<double *>(b + 8 * kSpMaxSorted)),
          cum(reinterpret_cast<double *>(b + 16 * kSpMaxSorted)),
          lg(reinterpret_cast<double *>(b + 24 * kSpMaxSorted)),
          ids(reinterpret_cast<int *>(b + 32 * kSpMaxSorted)),
          vals(reinterpret_cast<double *>(b + 36 * kSpMaxSorted)),
          pre(reinterpret_cast<double *>(b + 36 * kSpMaxSorted + 8 * kMaxGridCtas)) {}
};
constexpr size_t kSpScratchBytes = 36 * kSpMaxSorted + 8 * (2 * kMaxGridCtas + 1);
static_assert(kSpScratchBytes <= 8 * kSpBins, "the last CTA's scratch fits the histogram space");

// Inclusive prefix sum of the 64 entries a warp holds (lane l: entries l and l + 32).
__device__ __forceinline__ void warp_cum64(const double (&w)[2], double (&cum)[2]) {
    const int lane = threadIdx.x & 31;
    cum[0] = warp_incl_scan(w[0], lane);
    const double t0 = __shfl_sync(0xffffffffu, cum[0], 31);
    cum[1] = warp_incl_scan(w[1], lane) + t0;
}

// First entry (of 64) whose flag is set, or 64.
__device__ __forceinline__ int warp_first64(bool f0, bool f1) {
    const unsigned b0 = __ballot_sync(0xffffffffu, f0), b1 = __ballot_sync(0xffffffffu, f1);
    return b0 ? __ffs(b0) - 1 : (b1 ? 32 + __ffs(b1) - 1 : 64);
}
// Last entry (of 64) whose flag is set, or -1.
__device__ __forceinline__ int warp_last64(bool f0, bool f1) {
    const unsigned b0 = __ballot_sync(0xffffffffu, f0), b1 = __ballot_sync(0xffffffffu, f1);
    return b1 ? 63 - __clz(b1) : (b0 ? 31 - __clz(b0) : -1);
}

// A list of at most 64 entries finished by warp 0 alone (no CTA barriers): the keys sorted in
// descending order, the top-p cut, the id order when there is no cut, the draw.  Same arithmetic
// as the CTA-wide finish (prefix sums in another order: differences at rounding level only).
__device__ int sp_list_finish_warp(const SpParams &p, int n) {
    const int lane = threadIdx.x & 31, L = p.list_n;
    unsigned long long x[2] = {lane < n ? __ldcg(p.cand + lane) : 0ull, lane + 32 < n ? __ldcg(p.cand + lane + 32) : 0ull};
    // bitonic sort of the 64 keys, descending (entry e = lane + 32 h)
#pragma unroll
    for (int size = 2; size <= 64; size <<= 1) {
#pragma unroll
        for (int j = size >> 1; j > 0; j >>= 1) {
            if (j == 32) {
                if (x[0] < x[1]) {
                    const unsigned long long t = x[0];
                    x[0] = x[1];
                    x[1] = t;
                }
            } else {
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int e = lane + 32 * h;
                    const unsigned long long y = __shfl_xor_sync(0xffffffffu, x[h], j);
                    const bool lower = (e & j) == 0, desc = (e & size) == 0;
                    const unsigned long long hi = x[h] > y ? x[h] : y, lo = x[h] > y ? y : x[h];
                    x[h] = (desc == lower) ? hi : lo;
                }
            }
        }
    }
    const double l0 = __shfl_sync(0xffffffffu, sp_logit(x[0]), 0);
    double lg[2];
    int ids[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        lg[h] = sp_logit(x[h]);
        ids[h] = sp_id(x[h]);
    }
    int m = L;
    if (p.sorted) {
        double w[2], cum[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) w[h] = lane + 32 * h < L ? exp(lg[h] - l0) : 0.0;
        warp_cum64(w, cum);
        const double S = __shfl_sync(0xffffffffu, cum[1], 31);
        const double threshold = S * p.top_p;
        const int first = warp_first64(lane < L && cum[0] >= threshold, lane + 32 < L && cum[1] >= threshold);
        m = first < L ? first + 1 : L;
    } else {
        // the top L by ascending id: sort (id << 32 | float bits), complemented, descending
        unsigned long long z[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint32_t o = (uint32_t)(x[h] >> kSpIdBits);
            const uint32_t bits = (o & 0x80000000u) ? (o & 0x7FFFFFFFu) : ~o;
            z[h] = lane + 32 * h < L ? ~(((unsigned long long)ids[h] << 32) | bits) : 0ull;
        }
#pragma unroll
        for (int size = 2; size <= 64; size <<= 1) {
#pragma unroll
            for (int j = size >> 1; j > 0; j >>= 1) {
                if (j == 32) {
                    if (z[0] < z[1]) {
                        const unsigned long long t = z[0];
                        z[0] = z[1];
                        z[1] = t;
                    }
                } else {
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int e = lane + 32 * h;
                        const unsigned long long y = __shfl_xor_sync(0xffffffffu, z[h], j);
                        const bool lower = (e & j) == 0, desc = (e & size) == 0;
                        const unsigned long long hi = z[h] > y ? z[h] : y, lo = z[h] > y ? y : z[h];
                        z[h] = (desc == lower) ? hi : lo;
                    }
                }
            }
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const unsigned long long v = ~z[h];
            lg[h] = (double)__uint_as_float((uint32_t)v);
            ids[h] = (int)(v >> 32);
        }
    }
    double w[2], cum[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) w[h] = lane + 32 * h < m ? exp((lg[h] - l0) / p.temperature) : 0.0;
    warp_cum64(w, cum);
    const double total = __shfl_sync(0xffffffffu, cum[1], 31);
    const double sample = p.u * total;
    int pick = warp_first64(w[0] > 0.0 && sample < cum[0], w[1] > 0.0 && sample < cum[1]);
    if (pick >= m) pick = warp_last64(w[0] > 0.0, w[1] > 0.0);
    const int tok = pick < 32 ? __shfl_sync(0xffffffffu, ids[0], pick & 31) : __shfl_sync(0xffffffffu, ids[1], pick & 31);
    if (lane == 0) p.token[0] = tok;
    return MMRS_OK;
}

// The last CTA's part of a list call: the (at most 1024) appended keys sorted, the top list_n
// kept; with top-p, cut where the cumulative weight exp(l - max) reaches top_p of the total;
// without, visited by ascending id; then one draw.  Returns the status; writes the token.
__device__ int sp_list_finish(const SpParams &p, SpShared &s, unsigned char *scratch) {
    const int tid = threadIdx.x;
    SpScratch b(scratch);
    const int n = (int)__ldcg(&p.misc->ncand), L = p.list_n;
    if (n < L || n > kSpMaxSorted || L < 1) return MMRS_ERR_LAUNCH;  // the selection yields list_n..1024 keys
    int n2 = 2;
    while (n2 < n) n2 <<= 1;
    for (int i = tid; i < kSpMaxSorted; i += kSpThreads) b.sk[i] = i < n ? __ldcg(p.cand + i) : 0ull;
    __syncthreads();
    if (n2 <= 64)
        sp_warp_sort64_desc(b.sk, n);
    else
        sp_sort_desc(b.sk, n2);
    const double l0 = sp_logit(b.sk[0]);
    int m = L;
    if (p.sorted) {
        // top-p over weights at temperature 1 (exponential_weights(&candidates, 1.0)), sorted order
        for (int i = tid; i < kSpMaxSorted; i += kSpThreads) {
            const bool in = i < L;
            b.lg[i] = in ? sp_logit(b.sk[i]) : 0.0;
            b.ids[i] = in ? sp_id(b.sk[i]) : 0;
            b.w[i] = in ? exp(b.lg[i] - l0) : 0.0;
        }
        __syncthreads();
        double tot;
        sp_cumulate(b.w, b.cum, s, &tot);
        if (p.s_from_partials) sp_cta_prefix(p, s, b.vals, b.pre);
        const double S = p.s_from_partials ? b.pre[gridDim.x] : tot;
        const double threshold = S * p.top_p;
        if (tid == 0) s.first = kSpMaxSorted;
        __syncthreads();
        for (int i = tid; i < L; i += kSpThreads)
            if (b.cum[i] >= threshold) atomicMin(&s.first, i);
        __syncthreads();
        if (s.first >= L) {
            if (p.s_from_partials) return MMRS_ERR_UNSUPPORTED;  // the nucleus is longer than the list
            m = L;  // (rounding between the two sums: the whole list is the nucleus)
        } else {
            m = s.first + 1;
        }
    } else {
        // the top list_n by ascending id: sort (id << 32 | float bits), complemented, descending
        for (int i = tid; i < n2; i += kSpThreads) {
            const unsigned long long k = b.sk[i];
            const uint32_t o = (uint32_t)(k >> kSpIdBits);
            const uint32_t bits = (o & 0x80000000u) ? (o & 0x7FFFFFFFu) : ~o;
            b.sk[i] = i < L ? ~(((unsigned long long)sp_id(k) << 32) | bits) : 0ull;
        }
        __syncthreads();
        if (n2 <= 64)
            sp_warp_sort64_desc(b.sk, L);
        else
            sp_sort_desc(b.sk, n2);
        for (int i = tid; i < kSpMaxSorted; i += kSpThreads) {
            const bool in = i < L;
            const unsigned long long x = ~b.sk[i];
            b.lg[i] = in ? (double)__uint_as_float((uint32_t)x) : 0.0;
            b.ids[i] = in ? (int)(x >> 32) : 0;
        }
        __syncthreads();
    }
    // one draw over the first m entries at the requested temperature
    for (int i = tid; i < kSpMaxSorted; i += kSpThreads) b.w[i] = i < m ? exp((b.lg[i] - l0) / p.temperature) : 0.0;
    __syncthreads();
    double total;
    sp_cumulate(b.w, b.cum, s, &total);
    const double sample = p.u * total;
    if (tid == 0) {
        s.first = kSpMaxSorted;
        s.last = 0;
    }
    __syncthreads();
    for (int i = tid; i < m; i += kSpThreads) {
        if (b.w[i] > 0.0) {
            if (sample < b.cum[i]) atomicMin(&s.first, i);
            atomicMax(&s.last, i);
        }
    }
    __syncthreads();
    const int pick = s.first < m ? s.first : s.last;
    if (tid == 0) p.token[0] = b.ids[pick];
    return MMRS_OK;
}

__global__ void __launch_bounds__(kSpThreads, 1) sample_kernel(const SpParams p) {
    extern __shared__ __align__(16) unsigned char sp_smem[];
    __shared__ SpShared s;
    const int tid = threadIdx.x, lane = tid & 31, G = (int)gridDim.x, cta = (int)blockIdx.x;
    unsigned long long *keys = reinterpret_cast<unsigned long long *>(sp_smem);
    uint32_t *sh = reinterpret_cast<uint32_t *>(sp_smem + (size_t)8 * p.chunk);  // [2][kSpBins]
    unsigned char *scratch = sp_smem + (size_t)8 * p.chunk;                       // the same space, later
    const uint64_t deadline = globaltimer_ns() + kSpTimeoutNs;
    const int lo = min(p.V, cta * p.chunk), n = min(p.V, lo + p.chunk) - lo;
    if (tid == 0) {
        s.ok = 1;
        s.epoch = __ldcg(&p.ctl->epoch[cta]);
        s.max_key = 0ull;
        s.gmax_key = 0ull;
        s.flags = 0u;
    }
    int nsync = 0, rounds = 0;
    double gmax = 0.0;

    if (p.mode == kGreedy) {
        unsigned long long best = 0ull;
        for (int i = tid; i < n; i += kSpThreads) {
            const unsigned long long k = lm_key(__ldg(p.logits + lo + i), lo + i);
            best = k > best ? k : best;
        }
        best = warp_max_u64(best);
        __syncthreads();
        if (lane == 0 && best) atomicMax(&s.max_key, best);
        __syncthreads();
        if (tid == 0 && s.max_key) atomicMax(&p.misc->best, s.max_key);
    } else {
        // ---- phase 0: keys, non-finite values, largest key, round-0 histogram ----------------
        bool act[2] = {p.mode != kLogprob && p.kA > 0, p.mode != kLogprob && p.kB > 0};
        const bool select = act[0] || act[1];
        unsigned long long prefix[2] = {0ull, 0ull}, bound[2] = {0ull, 0ull};
        uint32_t need[2] = {(uint32_t)p.kA, (uint32_t)p.kB}, gt[2] = {0u, 0u};
        const int nb = act[1] ? 2 * kSpBins : kSpBins;  // (search B runs only beside A)
        if (select)
            for (int b = tid; b < nb; b += kSpThreads) sh[b] = 0u;
        __syncthreads();
        int nonfin = 0;
        unsigned long long kmax = 0ull;
        for (int i = tid; i < n; i += kSpThreads) {
            const float v = __ldg(p.logits + lo + i);
            nonfin |= (__float_as_uint(v) & 0x7F800000u) == 0x7F800000u;
            const unsigned long long key =
                ((unsigned long long)sp_order(v) << kSpIdBits) | (unsigned long long)(kSpIdMask - (uint32_t)(lo + i));
            keys[i] = key;
            kmax = key > kmax ? key : kmax;
            if (select) {
#pragma unroll
                for (int q = 0; q < 2; ++q)
                    if (act[q]) atomicAdd(&sh[q * kSpBins + (int)(key >> ((kSpRounds - 1) * kSpDigitBits))], 1u);
            }
        }
        kmax = warp_max_u64(kmax);
        if (lane == 0 && kmax) atomicMax(&s.max_key, kmax);
        if (__syncthreads_or(nonfin) && tid == 0) atomicOr(&p.misc->flags, kFlagNonfinite);
        if (tid == 0) p.cta_max[cta] = s.max_key;
        if (select) {
            for (int b = tid; b < nb; b += kSpThreads)
                if (sh[b]) atomicAdd(&p.hist[b], sh[b]);
            rounds = 1;
        }
        if (!sp_grid_sync(p, s, nsync, deadline)) return;

        // ---- global maximum and the call's flags (the same in every CTA) ----------------------
        {
            if (tid == 0) s.flags = __ldcg(&p.misc->flags);
            unsigned long long m = 0ull;
            for (int c = tid; c < G; c += kSpThreads) {
                const unsigned long long v = __ldcg(p.cta_max + c);
                m = v > m ? v : m;
            }
            m = warp_max_u64(m);
            if (lane == 0 && m) atomicMax(&s.gmax_key, m);
        }
        __syncthreads();
        gmax = sp_logit(s.gmax_key);
        const bool skip = p.mode != kLogprob && (s.flags & kFlagNonfinite);

        if (p.mode == kLogprob) {
            double acc = 0.0;
            for (int i = tid; i < n; i += kSpThreads) acc += exp(sp_logit(keys[i]) - gmax);
            double tot;
            block_excl_scan(acc, s.sw_d, tot);
            if (tid == 0) p.partial[cta] = tot;
        } else if (!skip) {
            // ---- radix selection ------------------------------------------------------------------
            bool failed = false;
            for (int r = 0; r < kSpRounds && (act[0] || act[1]); ++r) {
                if (r > 0) {
                    sp_histogram(p, keys, n, sh, r, prefix, act);
                    if (!sp_grid_sync(p, s, nsync, deadline)) return;
                    rounds = r + 1;
                    // every CTA has scanned round r - 1's histogram: clear this CTA's share of it
                    uint32_t *prev = p.hist + (size_t)(r - 1) * 2 * kSpBins;
                    const int per = (2 * kSpBins + G - 1) / G;
                    for (int b = cta * per + tid; b < min(2 * kSpBins, (cta + 1) * per); b += kSpThreads)
                        prev[b] = 0u;
                }
                const int shift = (kSpRounds - 1 - r) * kSpDigitBits;
                for (int q = 0; q < 2; ++q) {
                    if (!act[q]) continue;
                    uint32_t above = 0, in_bin = 0;
                    const int d = sp_scan(p, s, r, q, need[q], &above, &in_bin);
                    if (d < 0) {
                        failed = true;
                        act[0] = act[1] = false;
                        if (tid == 0) atomicOr(&p.misc->flags, kFlagInternal);
                        break;
                    }
                    prefix[q] = (prefix[q] << kSpDigitBits) | (unsigned long long)d;
                    gt[q] += above;
                    need[q] -= above;
                    if (shift == 0) {
                        bound[q] = prefix[q];  // the exact key of rank k
                        act[q] = false;
                    } else if (q == 0 && p.mode == kList && gt[q] + in_bin <= (uint32_t)kSpMaxSorted) {
                        bound[q] = prefix[q] << shift;  // at most 1024 keys at or above: the list sorts them
                        act[q] = false;
                    }
                }
            }
            if (!failed && p.mode == kList) {
                // ---- append the list's keys; sum the whole candidate set when it is longer --------
                double acc = 0.0;
                for (int i = tid; i < n; i += kSpThreads) {
                    const unsigned long long key = keys[i];
                    if (key >= bound[0]) {
                        const uint32_t pos = atomicAdd(&p.misc->ncand, 1u);
                        if (pos < (uint32_t)kSpMaxSorted) p.cand[pos] = key;
                    }
                    if (p.s_from_partials && key >= bound[1]) acc += exp(sp_logit(key) - gmax);
                }
                if (p.s_from_partials) {
                    double tot;
                    block_excl_scan(acc, s.sw_d, tot);
                    if (tid == 0) p.partial[cta] = tot;
                }
            } else if (!failed) {
                // ---- kIdWalk: walk the candidates by ascending id across the CTAs ------------------
                const unsigned long long tA = bound[0];
                const int per = (n + kSpThreads - 1) / kSpThreads;
                const int i0 = min(n, tid * per), i1 = min(n, i0 + per);
                double acc = 0.0;
                for (int i = i0; i < i1; ++i)
                    if (keys[i] >= tA) acc += exp((sp_logit(keys[i]) - gmax) / p.temperature);
                double mine;
                const double ex = block_excl_scan(acc, s.sw_d, mine);
                if (tid == 0) p.partial[cta] = mine;
                if (!sp_grid_sync(p, s, nsync, deadline)) return;
                SpScratch b(scratch);
                sp_cta_prefix(p, s, b.vals, b.pre);
                const double before = b.pre[cta], after = b.pre[cta + 1], total = b.pre[G];
                const double sample = p.u * total;
                const bool owner = before <= sample && sample < after;
                const bool fallback = sample >= total && cta == s.last_nz;
                if (owner || fallback) {
                    if (tid == 0) {
                        s.first = kSpMaxSlice;
                        s.last = -1;
                    }
                    __syncthreads();
                    double run = ex;
                    for (int i = i0; i < i1; ++i) {
                        if (keys[i] < tA) continue;
                        const double wi = exp((sp_logit(keys[i]) - gmax) / p.temperature);
                        run += wi;
                        if (wi > 0.0) {
                            if (owner && sample < before + run) {
                                atomicMin(&s.first, i);
                                break;
                            }
                            atomicMax(&s.last, i);
                        }
                    }
                    __syncthreads();
                    const int pick = s.first < kSpMaxSlice ? s.first : s.last;
                    if (tid == 0 && pick >= 0) p.token[0] = lo + pick;
                }
            }
        }
    }

    // ---- every CTA arrives; the last one finishes the call and leaves the workspace clean ----
    __syncthreads();
    if (tid == 0) {
        p.ctl->epoch[cta] = s.epoch + (uint32_t)nsync;  // read again only by this CTA's next launch
        // release this CTA's writes (ordered before by the barrier), acquire the others'
        uint32_t t;
        asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;" : "=r"(t) : "l"(&p.misc->ticket) : "memory");
        s.is_last = t == (uint32_t)G - 1u;
        if (s.is_last) s.flags = __ldcg(&p.misc->flags);
    }
    __syncthreads();
    if (!s.is_last) return;
    __syncthreads();
    const uint32_t flags = s.flags;
    int result = MMRS_OK;
    if (p.mode == kGreedy) {
        if (tid == 0) {
            const unsigned long long b = __ldcg(&p.misc->best);
            p.token[0] = (int32_t)(0xFFFFFFFFu - (uint32_t)(b & 0xFFFFFFFFull));
        }
    } else if (flags & kFlagInternal) {
        result = MMRS_ERR_LAUNCH;
    } else if (p.mode == kLogprob) {
        SpScratch b(scratch);
        sp_cta_prefix(p, s, b.vals, b.pre);
        if (tid == 0) {
            const double lt = (double)__ldg(p.logits + p.token_id);
            const float v = (float)(lt - gmax - log(b.pre[G]));
            p.out[0] = v;
            s.status = isfinite(v) ? MMRS_OK : MMRS_ERR_NONFINITE;
        }
        __syncthreads();
        result = s.status;
    } else if (flags & kFlagNonfinite) {
        result = MMRS_ERR_NONFINITE;
    } else if (p.mode == kList) {
        const int n = (int)__ldcg(&p.misc->ncand);
        if (n <= 64 && n >= p.list_n && p.list_n >= 1) {
            if (tid < 32) {
                const int r = sp_list_finish_warp(p, n);
                if (tid == 0) s.status = r;
            }
            __syncthreads();
            result = s.status;
        } else {
            result = sp_list_finish(p, s, scratch);
        }
    }
    if (result != MMRS_OK && p.token && tid == 0) p.token[0] = -1;
    // leave the workspace clean: the histogram rounds not cleared on the way (the last one run;
    // all of them when the call stopped early), the list counter, flags, maximum, ticket
    if (rounds > 0) {
        const int r0 = flags ? 0 : rounds - 1, r1 = flags ? kSpRounds : rounds;
        for (int b = r0 * 2 * kSpBins + tid; b < r1 * 2 * kSpBins; b += kSpThreads) p.hist[b] = 0u;
    }
    __syncthreads();
    if (tid == 0) {
        p.misc->best = 0ull;
        p.misc->ncand = 0u;
        p.misc->flags = 0u;
        p.misc->result = (uint32_t)result;
        p.misc->ticket = 0u;  // (the next launch sees all of these: kernel boundary)
    }
}

int sp_launch(const SpParams &p, int grid, cudaStream_t stream) {
    const size_t smem = (size_t)8 * p.chunk + (size_t)8 * kSpBins;
    // the dynamic shared-memory limit is raised once per device (the attribute is per context);
    // call_once keeps concurrent host threads from racing on it
    static std::once_flag once[64];
    static cudaError_t set_rc[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return MMRS_ERR_LAUNCH;
    std::call_once(once[dev], [dev] {
        set_rc[dev] = cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)((size_t)8 * kSpMaxSlice + (size_t)8 * kSpBins));
    });
    if (set_rc[dev] != cudaSuccess) return MMRS_ERR_LAUNCH;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kSpThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, sample_kernel, p) == cudaSuccess ? MMRS_OK : MMRS_ERR_LAUNCH;
}

// One grid for every call on a device (the barrier's epoch words count on it): one CTA per SM.
int sp_grid() {
    static std::once_flag once[64];
    static int grids[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
    std::call_once(once[dev], [dev] {
        int sms = 0;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && sms > 0)
            grids[dev] = sms < kMaxGridCtas ? sms : kMaxGridCtas;
    });
    return grids[dev];
}

int sp_bind(SpParams &p, void *workspace, size_t workspace_bytes, int vocab, int *grid) {
    const SpLayout l = sp_layout();
    if (!workspace || workspace_bytes < l.total || ((uintptr_t)workspace & 255u)) return MMRS_ERR_ARG;
    const int g = sp_grid();
    if (g <= 0) return MMRS_ERR_LAUNCH;
    const int chunk = (vocab + g - 1) / g;
    if (chunk > kSpMaxSlice) return MMRS_ERR_UNSUPPORTED;
    uint8_t *ws = static_cast<uint8_t *>(workspace);
    p.V = vocab;
    p.chunk = chunk;
    p.ctl = reinterpret_cast<GridFlags *>(ws + l.ctl);
    p.misc = reinterpret_cast<SpMisc *>(ws + l.misc);
    p.cta_max = reinterpret_cast<unsigned long long *>(ws + l.cta_max);
    p.partial = reinterpret_cast<double *>(ws + l.partial);
    p.hist = reinterpret_cast<uint32_t *>(ws + l.hist);
    p.cand = reinterpret_cast<unsigned long long *>(ws + l.cand);
    *grid = g;
    return MMRS_OK;
}

}  // namespace
}  // namespace mmrs

using namespace mmrs;

extern "C" size_t mmrs_sample_workspace_bytes(int vocab) {
    if (vocab < 1 || vocab > MMRS_SAMPLE_MAX_VOCAB) return 0;
    return sp_layout().total;
}

extern "C" int mmrs_sample_workspace_status(const void *workspace) {
    if (!workspace) return MMRS_ERR_ARG;
    const SpLayout l = sp_layout();
    uint32_t st = 0, res = 0;
    const uint8_t *ws = static_cast<const uint8_t *>(workspace);
    if (cudaMemcpy(&st, ws + l.ctl, sizeof(st), cudaMemcpyDeviceToHost) != cudaSuccess) return MMRS_ERR_LAUNCH;
    if (st != MMRS_OK) return (int)st;
    if (cudaMemcpy(&res, ws + l.misc + offsetof(SpMisc, result), sizeof(res), cudaMemcpyDeviceToHost) != cudaSuccess)
        return MMRS_ERR_LAUNCH;
    return (int)res;
}

extern "C" int mmrs_sample_token(const float *logits, int vocab, const MmrsSamplingParams *params, double u,
                                 int32_t *token, void *workspace, size_t workspace_bytes, mmrs_stream_t stream) {
    if (!logits || !token || !params || vocab < 1 || vocab > MMRS_SAMPLE_MAX_VOCAB) return MMRS_ERR_ARG;
    const double T = params->temperature, top_p = params->top_p;
    // SamplingParams::validate (src/sampling.rs:31-39); the draw lies in [0, 1)
    if (!isfinite(T) || T < 0.0 || !isfinite(top_p) || top_p < 0.0 || top_p > 1.0) return MMRS_ERR_ARG;
    if (T > 0.0 && !(u >= 0.0 && u < 1.0)) return MMRS_ERR_ARG;
    SpParams p = {};
    int grid = 0;
    const int rc = sp_bind(p, workspace, workspace_bytes, vocab, &grid);
    if (rc != MMRS_OK) return rc;
    p.logits = logits;
    p.token = token;
    p.temperature = T;
    p.top_p = top_p;
    p.u = u;
    if (T == 0.0) {
        p.mode = kGreedy;
    } else {
        const int k = (params->top_k > 0 && params->top_k < vocab) ? params->top_k : vocab;
        const bool sorted = top_p < 1.0 && k > 1;
        if (sorted || k <= kSpMaxSorted) {
            p.mode = kList;
            p.sorted = sorted;
            p.list_n = k < kSpMaxSorted ? k : kSpMaxSorted;
            p.kA = p.list_n < vocab ? p.list_n : 0;
            p.s_from_partials = sorted && k > p.list_n;
            p.kB = (p.s_from_partials && k < vocab) ? k : 0;
        } else {
            p.mode = kIdWalk;
            p.kA = k < vocab ? k : 0;
        }
    }
    return sp_launch(p, grid, (cudaStream_t)stream);
}

extern "C" int mmrs_token_logprob(const float *logits, int vocab, int token_id, float *out, void *workspace,
                                  size_t workspace_bytes, mmrs_stream_t stream) {
    if (!logits || !out || vocab < 1 || vocab > MMRS_SAMPLE_MAX_VOCAB) return MMRS_ERR_ARG;
    if (token_id < 0 || token_id >= vocab) return MMRS_ERR_ARG;
    SpParams p = {};
    int grid = 0;
    const int rc = sp_bind(p, workspace, workspace_bytes, vocab, &grid);
    if (rc != MMRS_OK) return rc;
    p.logits = logits;
    p.out = out;
    p.mode = kLogprob;
    p.token_id = token_id;
    return sp_launch(p, grid, (cudaStream_t)stream);
}
