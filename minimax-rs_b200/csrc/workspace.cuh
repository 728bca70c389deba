// Workspace layout of the fused MoE block (shared by the entry points in api.cu and noalloc.cu).
#pragma once
#include <stddef.h>
#include <stdint.h>

#include "decode.cuh"
#include "../../include/minimax_moe.h"

namespace mmrs {

struct WsLayout {
    size_t ctl, trace, score, arec, total;
};

// [control block (DecodeCtl)] | trace | tagged score copies | tagged act records; all of it zero
// before first use
WsLayout ws_layout(int E, int I, int max_tokens);
void ws_bind(DecodeParams &p, uint8_t *ws, const WsLayout &l);
int validate_weights(const MmrsMoeWeights *w);
// Status of the last reference-ABI launcher on this host thread (read by mmrs_last_error()).
void record_error(int status);

}  // namespace mmrs
