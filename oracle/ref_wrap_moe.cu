// Test infrastructure: the reference's MoE launchers (moe/moe_gguf.cu, compiled from the reference
// tree by oracle/build_ref.sh) plus a launcher for its file-local quantize_q8_1 kernel
// (gguf.cuh:1234-1261) with the launch geometry the reference uses (moe_gguf.cu:368-377).
#include "moe_gguf.cu"

extern "C" int ref_quantize_q8_1(const float *x, void *out, int rows, int kx, int kx_padded, cudaStream_t s) {
    const int blocks = (kx_padded + CUDA_QUANTIZE_BLOCK_SIZE - 1) / CUDA_QUANTIZE_BLOCK_SIZE;
    quantize_q8_1<<<dim3(blocks, rows, 1), dim3(CUDA_QUANTIZE_BLOCK_SIZE, 1, 1), 0, s>>>(x, out, kx, kx_padded);
    return (int)cudaGetLastError();
}
