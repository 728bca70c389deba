// Test infrastructure: exposes the reference's own f32 k-quant dequantisers (compiled from the
// reference tree by oracle/build_ref.sh) with a launcher.  Launch geometry follows the kernels'
// own comments (quantized.cu:943, 985): one block per super-block, 32 threads for Q4_K and
// 64 for Q5_K.
#include "quantized.cu"

extern "C" int ref_dequant_q4k_f32(const void *blocks, float *out, int nblocks, cudaStream_t s) {
    dequantize_block_q4_K_f32<<<nblocks, 32, 0, s>>>(blocks, out);
    return (int)cudaGetLastError();
}
extern "C" int ref_dequant_q5k_f32(const void *blocks, float *out, int nblocks, cudaStream_t s) {
    dequantize_block_q5_K_f32<<<nblocks, 64, 0, s>>>(blocks, out);
    return (int)cudaGetLastError();
}
