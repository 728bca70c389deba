// Multi-token (prefill) MoE path: routing for T tokens, stable route bucketing, gathered Q8_1
// quantisation and a grouped expert GEMM on the 5th-generation tensor cores (tcgen05, kind::i8).
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace mmrs {

constexpr int kPfNT = 32;           // routes per GEMM tile (MMA N <= 32)
constexpr int kPfMT = 128;          // weight rows per GEMM tile (MMA M)
constexpr int kPfSegAlign = 16;     // each expert's route segment is padded to this many rows
constexpr int kPfRawStages = 3;     // raw GGUF weight tiles in flight (TMA)
constexpr int kPfOpStages = 3;      // unpacked operand stages (A int8, scales)
constexpr int kPfGroups = 2;        // TMEM groups: the 8 block accumulators of one chunk each
constexpr int kPfEpiWarps = 16;     // epilogue warps: 4 TMEM lane quarters x 4 units of 8 routes
constexpr int kPfUnpackWarps = 4;   // one thread per weight row
constexpr int kPfThreads = 32 * (2 + kPfUnpackWarps + kPfEpiWarps);  // TMA, MMA, unpack, epilogue
constexpr int kPfMaxExperts = 1024;

// Activation quantisation numerics.
enum PfMode : int {
    kPfModeMmq = 0,      // quantize_mmq_q8_1<DS4> + MMQ combine (mmq_quantize.cu:59-72, mmq_gguf.cuh)
    kPfModeGeneric = 1,  // quantize_q8_1 + vec_dot_q*_K_q8_1 combine (gguf.cuh:1234-1261, 727-842)
};

// Bucketing of routes by expert (device arrays).  Routes of expert e occupy padded rows
// [seg[e], seg[e] + count[e]) of the gathered activation matrix; seg[e] is a multiple of 16.
struct PfPlan {
    int *count;      // [E]
    int *first;      // [E] first position of expert e in the expert-sorted route list
    int *seg;        // [E]
    int *tiles;      // [E + 1] exclusive prefix of ceil(count / kPfNT); tiles[E] = total
    int *row_route;  // [ppad] route id of each padded row, -1 for padding
    int ppad;        // row capacity: routes + (kPfSegAlign - 1) * E, rounded up to kPfSegAlign
};

__host__ __device__ inline int pf_ppad(int routes, int E) {
    return pad_to(routes + (kPfSegAlign - 1) * E, kPfSegAlign);
}

// Gathered, quantised activations in the tensor-core operand layout.  For padded row p and
// column k (k < K, K a multiple of 256), the int8 lives at
//   (k / 256) * ppad * 256 + (p / 8) * 2048 + ((k % 256) / 16) * 128 + (p % 8) * 16 + k % 16
// i.e. per 256-column chunk, 8-row groups of sixteen 8x16-byte core matrices (the canonical
// no-swizzle K-major layout of a UMMA operand).  The block scales of 16 consecutive rows form one
// 1 KiB record per chunk, d8 plane then s8 plane:
//   ds[((k / 256) * (ppad / 16) + p / 16) * 256 + plane * 128 + ((k % 256) / 32) * 16 + p % 16]
struct PfActs {
    int8_t *q;
    float *ds;
};

struct PfGemmParams {
    const int8_t *aq;
    const float *ads;
    PfPlan plan;
    const float *route_scale;  // nullable: output row of route r is multiplied by route_scale[r]
    float *out;                // [routes][N], row = route id
    int E, N, K, gtype, mode, mt;
    uint32_t *status;          // device error word (MMRS_ERR_TIMEOUT on an expired wait)
    uint64_t timeout_ns;
};

// Host launchers (all asynchronous on `stream`; return an MMRS status).
int pf_router_logits(const float *x, const float *router, int T, int E, int H, float *logits, cudaStream_t s);
int pf_route_topk(const float *logits, const float *bias, int T, int E, uint32_t *ids, float *w,
                  cudaStream_t s);
int pf_sort_routes(const uint32_t *keys, int n, int end_bit, uint32_t *sorted_keys, uint32_t *sorted_routes,
                   cudaStream_t s);
// Experts with e % own_world != own_rank are left out of the plan (expert parallel); own_world = 1
// keeps every expert.
int pf_build_plan(const int32_t *sorted_experts, const int32_t *sorted_routes, int M, int E, PfPlan plan,
                  cudaStream_t s, int own_world = 1, int own_rank = 0);
// Quantise the gathered input rows: padded row p takes input row route / div (x) or, with x2,
// the product x2 * silu(x) of route rows (silu = x / (1 + exp(-x))).
int pf_quantize(const float *x, const float *x2, int div, int K, int mode, PfPlan plan, PfActs acts, int rows_max,
                cudaStream_t s);
int pf_gemm(const void *weights, PfGemmParams p, int rows_max, cudaStream_t s);
// y[t] = sum over the token's 8 routes (ascending) of dn[route] (+ residual); with own_world > 1 only
// the routes whose expert (ids) satisfies e % own_world == own_rank are summed.
int pf_reduce_topk(const float *dn, const float *residual, int T, int H, float *y, cudaStream_t s,
                   const uint32_t *ids = nullptr, int own_world = 1, int own_rank = 0);
size_t pf_gemm_smem_bytes();

}  // namespace mmrs
