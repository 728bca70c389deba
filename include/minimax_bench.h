/* Measurement helpers of minimax-rs B200 (no counterpart in the reference): the measured
 * denominators of the roofline fractions the benchmark reports. */
#ifndef MINIMAX_BENCH_H
#define MINIMAX_BENCH_H

#include "minimax_moe.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Dense int8 tensor-core throughput of the current device in TOPS (2 ops a multiply-add): every
 * SM issues chunks * 8 back-to-back tcgen05.mma.kind::i8 of M = 128, N = 256, K = 32 from shared
 * memory into TMEM; the best of `reps` event-timed launches (after one warm-up) is reported.
 * chunks = 4096 runs ~2 ms a launch on a B200. */
MMRS_API int mmrs_int8_tensor_peak(int chunks, int reps, double *tops, mmrs_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif
