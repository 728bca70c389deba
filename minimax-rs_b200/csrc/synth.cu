// Seeded synthetic inputs for tests and the benchmark, generated on the device so that full-size
// expert tensors (2.2 GB per layer) never cross PCIe.  The generator is a pure function of
// (seed, stream id, element index) and is mirrored bit-for-bit by minimax-rs_b200/synth.py.
//
//   mix64      : SplitMix64 output function (Steele, Lea & Flood 2014)
//   key        : mix64(seed * G ^ (stream + 1) * C)
//   rand64(i)  : mix64(key + (i + 1) * G)
//   normal(i)  : Irwin-Hall sum of the eight 16-bit fields of rand64(2i), rand64(2i+1),
//                centred and scaled to unit variance (exact integer sum, one f32 multiply).
#include "common.cuh"

namespace mmrs {

constexpr uint64_t kGolden = 0x9E3779B97F4A7C15ull;
constexpr uint64_t kStreamMul = 0xD1B54A32D192ED03ull;
constexpr uint32_t kInvStdBits = 0x379cc471u;  // f32(1 / (65536 * sqrt(2/3)))

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
__device__ __forceinline__ uint64_t stream_key(uint64_t seed, uint32_t stream) {
    return mix64((seed * kGolden) ^ (((uint64_t)stream + 1ull) * kStreamMul));
}
__device__ __forceinline__ uint64_t rand64(uint64_t key, uint64_t i) { return mix64(key + (i + 1ull) * kGolden); }
__device__ __forceinline__ float synth_normal(uint64_t key, uint64_t i) {
    const uint64_t a = rand64(key, 2 * i), b = rand64(key, 2 * i + 1);
    int s = 0;
#pragma unroll
    for (int f = 0; f < 4; ++f) s += (int)((a >> (16 * f)) & 0xffffu) + (int)((b >> (16 * f)) & 0xffffu);
    return __fmul_rn((float)(s - 262140), __uint_as_float(kInvStdBits));
}
__device__ __forceinline__ float round_bf16(float v) {
    uint32_t b = __float_as_uint(v);
    b += 0x7fffu + ((b >> 16) & 1u);
    return __uint_as_float(b & 0xffff0000u);
}

__global__ void synth_normal_kernel(float *dst, int64_t n, uint64_t key, float scale, int bf16) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        float v = __fmul_rn(synth_normal(key, (uint64_t)i), scale);
        dst[i] = bf16 ? round_bf16(v) : v;
    }
}

// One thread per 8-byte word of the output window.
__global__ void synth_kquant_kernel(uint64_t *dst, uint64_t key, uint64_t key_d, int words_per_block,
                                    int rows, int nblk_total, int row0, int nrows, int kblk0, int nkblk,
                                    int64_t total_words) {
    for (int64_t w = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; w < total_words;
         w += (int64_t)gridDim.x * blockDim.x) {
        const int j = (int)(w % words_per_block);
        const int64_t blk_local = w / words_per_block;
        const int b = (int)(blk_local % nkblk);
        const int64_t er = blk_local / nkblk;  // expert * nrows + r
        const int r = (int)(er % nrows);
        const int64_t e = er / nrows;
        const int64_t gblk = (e * rows + row0 + r) * (int64_t)nblk_total + kblk0 + b;
        uint64_t v = rand64(key, (uint64_t)(gblk * words_per_block + j));
        if (j == 0) {
            const float d = __fmul_rn(fabsf(synth_normal(key_d, (uint64_t)(2 * gblk))), 0.01f);
            const float dm = __fmul_rn(fabsf(synth_normal(key_d, (uint64_t)(2 * gblk + 1))), 0.01f);
            const uint64_t hd = __half_as_ushort(__float2half_rn(d));
            const uint64_t hm = __half_as_ushort(__float2half_rn(dm));
            v = (v & 0xffffffff00000000ull) | hd | (hm << 16);
        }
        dst[w] = v;
    }
}

}  // namespace mmrs

using namespace mmrs;

extern "C" int mmrs_synth_normal_f32(float *dst, int64_t n, uint64_t seed, uint32_t stream_id, float scale,
                                     int round_bf16_flag, mmrs_stream_t stream) {
    if (!dst || n < 0) return MMRS_ERR_ARG;
    if (n == 0) return MMRS_OK;
    uint64_t key;
    {
        // host copy of stream_key
        auto hmix = [](uint64_t z) {
            z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
            z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
            return z ^ (z >> 31);
        };
        key = hmix((seed * kGolden) ^ (((uint64_t)stream_id + 1ull) * kStreamMul));
    }
    const int threads = 256;
    const int64_t blocks64 = (n + threads - 1) / threads;
    const int blocks = (int)(blocks64 < 148 * 64 ? blocks64 : 148 * 64);
    synth_normal_kernel<<<blocks, threads, 0, (cudaStream_t)stream>>>(dst, n, key, scale, round_bf16_flag);
    return cudaGetLastError() == cudaSuccess ? MMRS_OK : MMRS_ERR_LAUNCH;
}

extern "C" int mmrs_synth_kquant(void *dst, int gguf_type, uint64_t seed, uint32_t stream_id, int experts,
                                 int rows, int k, int row0, int nrows, int kblk0, int nkblk,
                                 mmrs_stream_t stream) {
    if (!dst || (gguf_type != MMRS_Q4K && gguf_type != MMRS_Q5K)) return MMRS_ERR_ARG;
    if (k % QK_K || experts <= 0 || rows <= 0 || nrows <= 0 || nkblk <= 0) return MMRS_ERR_ARG;
    const int nblk_total = k / QK_K;
    if (row0 < 0 || row0 + nrows > rows || kblk0 < 0 || kblk0 + nkblk > nblk_total) return MMRS_ERR_ARG;
    if (((uintptr_t)dst) & 7) return MMRS_ERR_ARG;
    auto hmix = [](uint64_t z) {
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        return z ^ (z >> 31);
    };
    const uint64_t key = hmix((seed * kGolden) ^ (((uint64_t)stream_id + 1ull) * kStreamMul));
    const uint64_t key_d = hmix((seed * kGolden) ^ (((uint64_t)stream_id + 0x10000ull + 1ull) * kStreamMul));
    const int wpb = kq_block_bytes(gguf_type) / 8;
    const int64_t total = (int64_t)experts * nrows * nkblk * wpb;
    const int threads = 256;
    const int64_t blocks64 = (total + threads - 1) / threads;
    const int blocks = (int)(blocks64 < 148 * 64 ? blocks64 : 148 * 64);
    synth_kquant_kernel<<<blocks, threads, 0, (cudaStream_t)stream>>>((uint64_t *)dst, key, key_d, wpb, rows,
                                                                      nblk_total, row0, nrows, kblk0, nkblk, total);
    return cudaGetLastError() == cudaSuccess ? MMRS_OK : MMRS_ERR_LAUNCH;
}
