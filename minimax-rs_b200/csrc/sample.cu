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
//   rounds   radix selection of the k-th largest key, 13 bits a round (4 rounds, one grid barrier
//            each): every CTA adds its shared-memory histogram into a global one, and after the
//            barrier every CTA scans the same global histogram, so all agree on the next digit
//            without another exchange.  Two ranks are selected side by side when needed (the
//            list top-p sorts, and the whole candidate set when top_k is larger than the list);
//   top-p    CTAs append the keys at or above the list's threshold (at most 1024) to a global
//            list; the last CTA to finish sorts it (bitonic, shared memory), cuts it where the
//            cumulative weight reaches top_p of the total and draws from what is left;
//   no top-p every CTA sums the weights of its slice's candidates (ids ascending), one more
//            barrier lets every CTA form the same prefix over CTAs, and the CTA whose range holds
//            u * total walks its slice to the chosen id.
// Weights and sums are double, as the reference's.  The grid barrier is the bounded software
// barrier of common.cuh (epoch words in the workspace); nothing else waits.
#include <cuda_runtime.h>
#include <math.h>
#include <stddef.h>

#include "../../include/minimax_sample.h"
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

enum SpMode : int { kGreedy = 0, kSorted = 1, kIdOrder = 2, kLogprob = 3 };

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
    int list_n;           // kSorted: length of the sorted list (min(top_k, 1024))
    int s_from_partials;  // top-p total over a candidate set larger than the sorted list
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
    unsigned long long max_key;
    double d[4];
    int i[8];
    int ok;
    uint32_t epoch;
};

// Histogram of round r for the active searches over the CTA's keys, added into the global one.
__device__ void sp_histogram(const SpParams &p, const unsigned long long *keys, int n, uint32_t *sh, int r,
                             const unsigned long long *prefix, const bool *act) {
    const int tid = threadIdx.x;
    const int shift = (kSpRounds - 1 - r) * kSpDigitBits;
    for (int b = tid; b < 2 * kSpBins; b += kSpThreads) sh[b] = 0u;
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
    for (int b = tid; b < 2 * kSpBins; b += kSpThreads)
        if (act[b / kSpBins] && sh[b]) atomicAdd(&gh[b], sh[b]);
}

// Digit of round r for search s: the largest d with (count in bins above d) < need; returns the
// count above it through *above (-1 digit when the histogram holds fewer than `need` keys).
__device__ int sp_scan(const SpParams &p, SpShared &s, int r, int srch, uint32_t need, uint32_t *above) {
    const int tid = threadIdx.x;
    const uint32_t *gh = p.hist + ((size_t)r * 2 + srch) * kSpBins;
    const int top = kSpBins - 1 - tid * kSpBinsPerThread;  // this thread: digits top, top-1, ...
    uint32_t c[kSpBinsPerThread];
    uint32_t sum = 0;
#pragma unroll
    for (int j = 0; j < kSpBinsPerThread; ++j) {
        c[j] = __ldcg(gh + top - j);
        sum += c[j];
    }
    if (tid == 0) s.i[2] = -1;
    uint32_t tot;
    const uint32_t ex = block_excl_scan(sum, s.sw_u, tot);  // (its barriers order the store above)
    if (ex < need && need <= ex + sum) {
        uint32_t run = ex;
#pragma unroll
        for (int j = 0; j < kSpBinsPerThread; ++j) {
            if (run + c[j] >= need) {
                s.i[2] = top - j;
                s.i[3] = (int)run;
                break;
            }
            run += c[j];
        }
    }
    __syncthreads();
    const int d = s.i[2];
    *above = (uint32_t)s.i[3];
    __syncthreads();  // (the next scan resets s.i[2])
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

// Inclusive cumulative weights of the sorted list (two entries per thread: 2t, 2t + 1).
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

// The last CTA's part of a top-p call: sort, cut, draw.  Returns the status; writes *token.
__device__ int sp_sorted_finish(const SpParams &p, SpShared &s, unsigned char *scratch) {
    const int tid = threadIdx.x;
    unsigned long long *sk = reinterpret_cast<unsigned long long *>(scratch);   // [1024]
    double *w = reinterpret_cast<double *>(scratch + 8 * kSpMaxSorted);         // [1024]
    double *cum = reinterpret_cast<double *>(scratch + 16 * kSpMaxSorted);      // [1024]
    const int n = min((int)__ldcg(&p.misc->ncand), kSpMaxSorted);
    if (n != p.list_n || n < 1) return MMRS_ERR_LAUNCH;  // the selection always yields list_n keys
    int n2 = 2;
    while (n2 < n) n2 <<= 1;
    for (int i = tid; i < kSpMaxSorted; i += kSpThreads) sk[i] = i < n ? __ldcg(p.cand + i) : 0ull;
    __syncthreads();
    sp_sort_desc(sk, n2);
    const double l0 = sp_logit(sk[0]);
    // top-p over weights at temperature 1 (exponential_weights(&candidates, 1.0))
    for (int i = tid; i < kSpMaxSorted; i += kSpThreads) w[i] = i < n ? exp(sp_logit(sk[i]) - l0) : 0.0;
    __syncthreads();
    double tot;
    sp_cumulate(w, cum, s, &tot);
    if (p.s_from_partials && tid == 0) {
        double S = 0.0;
        for (int c = 0; c < (int)gridDim.x; ++c) S += __ldcg(p.partial + c);
        s.d[0] = S;
    }
    if (tid == 0) s.i[4] = kSpMaxSorted;
    __syncthreads();
    const double S = p.s_from_partials ? s.d[0] : tot;
    const double threshold = S * p.top_p;
    for (int i = tid; i < n; i += kSpThreads)
        if (cum[i] >= threshold) atomicMin(&s.i[4], i);
    __syncthreads();
    int m = s.i[4] + 1;
    if (s.i[4] >= n) {
        if (p.s_from_partials) return MMRS_ERR_UNSUPPORTED;  // the nucleus is longer than the list
        m = n;  // (rounding between the two sums; the whole list is the nucleus)
    }
    // draw over the nucleus at the requested temperature
    __syncthreads();
    for (int i = tid; i < kSpMaxSorted; i += kSpThreads)
        w[i] = i < m ? exp((sp_logit(sk[i]) - l0) / p.temperature) : 0.0;
    __syncthreads();
    double total;
    sp_cumulate(w, cum, s, &total);
    const double sample = p.u * total;
    if (tid == 0) {
        s.i[5] = kSpMaxSorted;
        s.i[6] = 0;
    }
    __syncthreads();
    for (int i = tid; i < m; i += kSpThreads) {
        if (w[i] > 0.0) {
            if (sample < cum[i]) atomicMin(&s.i[5], i);
            atomicMax(&s.i[6], i);
        }
    }
    __syncthreads();
    const int pick = s.i[5] < m ? s.i[5] : s.i[6];
    if (tid == 0) p.token[0] = sp_id(sk[pick]);
    return MMRS_OK;
}

__global__ void __launch_bounds__(kSpThreads, 1) sample_kernel(const SpParams p) {
    extern __shared__ __align__(16) unsigned char sp_smem[];
    __shared__ SpShared s;
    const int tid = threadIdx.x, lane = tid & 31, G = (int)gridDim.x, cta = (int)blockIdx.x;
    unsigned long long *keys = reinterpret_cast<unsigned long long *>(sp_smem);
    uint32_t *sh = reinterpret_cast<uint32_t *>(sp_smem + (size_t)8 * p.chunk);  // [2][kSpBins]
    const uint64_t deadline = globaltimer_ns() + kSpTimeoutNs;
    const int lo = min(p.V, cta * p.chunk), n = min(p.V, lo + p.chunk) - lo;
    if (tid == 0) {
        s.ok = 1;
        s.epoch = __ldcg(&p.ctl->epoch[cta]);
        s.max_key = 0ull;
    }
    int nsync = 0;
    bool skip = false;

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
        // ---- phase 0: keys, non-finite values, largest key, round-0 histogram --------------
        const bool select = p.mode != kLogprob && (p.kA > 0 || p.kB > 0);
        const bool act[2] = {p.kA > 0, p.kB > 0};
        unsigned long long prefix[2] = {0ull, 0ull};
        uint32_t need[2] = {(uint32_t)p.kA, (uint32_t)p.kB};
        if (select)
            for (int b = tid; b < 2 * kSpBins; b += kSpThreads) sh[b] = 0u;
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
            for (int b = tid; b < 2 * kSpBins; b += kSpThreads)
                if (act[b / kSpBins] && sh[b]) atomicAdd(&p.hist[b], sh[b]);
        }
        if (!sp_grid_sync(p, s, nsync, deadline)) return;

        // ---- global maximum and the call's flags (the same in every CTA) --------------------
        if (tid == 0) s.max_key = 0ull;
        __syncthreads();
        {
            unsigned long long m = 0ull;
            for (int c = tid; c < G; c += kSpThreads) {
                const unsigned long long v = __ldcg(p.cta_max + c);
                m = v > m ? v : m;
            }
            m = warp_max_u64(m);
            if (lane == 0 && m) atomicMax(&s.max_key, m);
        }
        __syncthreads();
        const double gmax = sp_logit(s.max_key);
        if (p.mode != kLogprob && (__ldcg(&p.misc->flags) & kFlagNonfinite)) skip = true;

        if (p.mode == kLogprob) {
            double acc = 0.0;
            for (int i = tid; i < n; i += kSpThreads) acc += exp(sp_logit(keys[i]) - gmax);
            double tot;
            block_excl_scan(acc, s.sw_d, tot);
            if (tid == 0) p.partial[cta] = tot;
        } else if (!skip) {
            // ---- radix selection --------------------------------------------------------------
            if (select) {
                for (int r = 0; r < kSpRounds && !skip; ++r) {
                    if (r > 0) {
                        sp_histogram(p, keys, n, sh, r, prefix, act);
                        if (!sp_grid_sync(p, s, nsync, deadline)) return;
                        // every CTA has scanned round r - 1's histogram: clear this CTA's share
                        uint32_t *prev = p.hist + (size_t)(r - 1) * 2 * kSpBins;
                        const int per = (2 * kSpBins + G - 1) / G;
                        for (int b = cta * per + tid; b < min(2 * kSpBins, (cta + 1) * per); b += kSpThreads)
                            prev[b] = 0u;
                    }
                    for (int q = 0; q < 2; ++q) {
                        if (!act[q]) continue;
                        uint32_t above = 0;
                        const int d = sp_scan(p, s, r, q, need[q], &above);
                        if (d < 0) {
                            skip = true;
                            if (tid == 0) atomicOr(&p.misc->flags, kFlagInternal);
                            break;
                        }
                        prefix[q] = (prefix[q] << kSpDigitBits) | (unsigned long long)d;
                        need[q] -= above;
                    }
                }
            }
            const unsigned long long tA = act[0] ? prefix[0] : 0ull, tB = act[1] ? prefix[1] : 0ull;
            if (!skip && p.mode == kSorted) {
                // ---- top-p: append the list's keys; sum the whole candidate set if needed ---------
                double acc = 0.0;
                for (int i = tid; i < n; i += kSpThreads) {
                    const unsigned long long key = keys[i];
                    if (key >= tA) {
                        const uint32_t pos = atomicAdd(&p.misc->ncand, 1u);
                        if (pos < (uint32_t)kSpMaxSorted) p.cand[pos] = key;
                    }
                    if (p.s_from_partials && key >= tB) acc += exp(sp_logit(key) - gmax);
                }
                if (p.s_from_partials) {
                    double tot;
                    block_excl_scan(acc, s.sw_d, tot);
                    if (tid == 0) p.partial[cta] = tot;
                }
            } else if (!skip) {
                // ---- no top-p: walk the candidates by ascending id -------------------------------
                const int per = (n + kSpThreads - 1) / kSpThreads;
                const int i0 = min(n, tid * per), i1 = min(n, i0 + per);
                double acc = 0.0;
                for (int i = i0; i < i1; ++i)
                    if (keys[i] >= tA) acc += exp((sp_logit(keys[i]) - gmax) / p.temperature);
                double mine;
                const double ex = block_excl_scan(acc, s.sw_d, mine);
                if (tid == 0) p.partial[cta] = mine;
                if (!sp_grid_sync(p, s, nsync, deadline)) return;
                if (tid == 0) {
                    double run = 0.0, before = 0.0;
                    int last_nz = -1;
                    for (int c = 0; c < G; ++c) {
                        const double v = __ldcg(p.partial + c);
                        if (c == cta) before = run;
                        if (v > 0.0) last_nz = c;
                        run += v;
                    }
                    s.d[0] = before;
                    s.d[1] = run;
                    s.i[0] = last_nz;
                    s.i[5] = kSpMaxSlice;
                    s.i[6] = -1;
                }
                __syncthreads();
                const double before = s.d[0], total = s.d[1], sample = p.u * total;
                const bool owner = mine > 0.0 && before <= sample && sample < before + mine;
                const bool fallback = sample >= total && cta == s.i[0];
                if (owner || fallback) {
                    double run = ex;
                    for (int i = i0; i < i1; ++i) {
                        if (keys[i] < tA) continue;
                        const double wi = exp((sp_logit(keys[i]) - gmax) / p.temperature);
                        run += wi;
                        if (wi > 0.0) {
                            if (owner && sample < before + run) {
                                atomicMin(&s.i[5], i);
                                break;
                            }
                            atomicMax(&s.i[6], i);
                        }
                    }
                    __syncthreads();
                    const int pick = s.i[5] < kSpMaxSlice ? s.i[5] : s.i[6];
                    if (tid == 0 && pick >= 0) p.token[0] = lo + pick;
                }
            }
        }
    }

    // ---- every CTA arrives; the last one finishes the call and leaves the workspace clean ----
    __syncthreads();
    if (tid == 0) {
        p.ctl->epoch[cta] = s.epoch + (uint32_t)nsync;  // read again only by this CTA's next launch
        __threadfence();
        s.i[7] = atomicAdd(&p.misc->ticket, 1u) == (uint32_t)G - 1u;
    }
    __syncthreads();
    if (!s.i[7]) return;
    __threadfence();
    int result = MMRS_OK;
    const uint32_t flags = __ldcg(&p.misc->flags);
    unsigned char *scratch = sp_smem + (size_t)8 * p.chunk;  // the histogram space, free now
    if (p.mode == kGreedy) {
        if (tid == 0) {
            const unsigned long long b = __ldcg(&p.misc->best);
            p.token[0] = (int32_t)(0xFFFFFFFFu - (uint32_t)(b & 0xFFFFFFFFull));
        }
    } else if (flags & kFlagInternal) {
        result = MMRS_ERR_LAUNCH;
    } else if (p.mode == kLogprob) {
        if (tid == 0) {
            double S = 0.0;
            for (int c = 0; c < G; ++c) S += __ldcg(p.partial + c);
            unsigned long long m = 0ull;
            for (int c = 0; c < G; ++c) {
                const unsigned long long v = __ldcg(p.cta_max + c);
                m = v > m ? v : m;
            }
            const double lt = (double)__ldg(p.logits + p.token_id);
            const float v = (float)(lt - sp_logit(m) - log(S));
            p.out[0] = v;
            s.i[1] = isfinite(v) ? MMRS_OK : MMRS_ERR_NONFINITE;
        }
        __syncthreads();
        result = s.i[1];
    } else if (flags & kFlagNonfinite) {
        result = MMRS_ERR_NONFINITE;
    } else if (p.mode == kSorted) {
        result = sp_sorted_finish(p, s, scratch);
    }
    if (result != MMRS_OK && p.token && tid == 0) p.token[0] = -1;
    // leave the workspace clean: the histograms not cleared on the way (round 3's; all of them
    // when the rounds stopped early), the list counter, flags, maximum, ticket
    if ((p.mode == kSorted || p.mode == kIdOrder) && (p.kA > 0 || p.kB > 0)) {
        const int r0 = flags ? 0 : kSpRounds - 1;
        for (int b = r0 * 2 * kSpBins + tid; b < kSpRounds * 2 * kSpBins; b += kSpThreads) p.hist[b] = 0u;
    }
    __syncthreads();
    if (tid == 0) {
        p.misc->best = 0ull;
        p.misc->ncand = 0u;
        p.misc->flags = 0u;
        p.misc->result = (uint32_t)result;
        __threadfence();
        p.misc->ticket = 0u;
    }
}

int sp_launch(const SpParams &p, int grid, cudaStream_t stream) {
    const size_t smem = (size_t)8 * p.chunk + (size_t)8 * kSpBins;
    static int configured[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || configured[dev] < (int)smem) {
        if (cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)((size_t)8 * kSpMaxSlice + (size_t)8 * kSpBins)) != cudaSuccess)
            return MMRS_ERR_LAUNCH;
        if (dev >= 0 && dev < 64) configured[dev] = (int)((size_t)8 * kSpMaxSlice + (size_t)8 * kSpBins);
    }
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
    static int grids[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    if (dev >= 0 && dev < 64 && grids[dev]) return grids[dev];
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) return 0;
    const int g = sms < kMaxGridCtas ? sms : kMaxGridCtas;
    if (dev >= 0 && dev < 64) grids[dev] = g;
    return g;
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
        if (top_p < 1.0 && k > 1) {
            p.mode = kSorted;
            p.list_n = k < kSpMaxSorted ? k : kSpMaxSorted;
            p.kA = p.list_n < vocab ? p.list_n : 0;
            p.s_from_partials = k > p.list_n;
            p.kB = (k > p.list_n && k < vocab) ? k : 0;
        } else {
            p.mode = kIdOrder;
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
