"""Python binding of the B200-native MiniMax-M2.7 MoE hot path (ctypes over the C ABI).

The compute lives in lib/libminimax_moe.so (hand-written sm_100a CUDA, see csrc/).  This module
only declares the C prototypes of include/minimax_moe.h and offers thin helpers that take torch
CUDA tensors.  There is no CPU fallback: every entry point raises when the library is missing.

The directory name contains a dash, so import it by path:

    import importlib.util, sys
    spec = importlib.util.spec_from_file_location("minimax_rs_b200", "<repo>/minimax-rs_b200/__init__.py",
                                                  submodule_search_locations=["<repo>/minimax-rs_b200"])
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
LIB_PATH = PKG_DIR / "lib" / "libminimax_moe.so"
HEADER = PKG_DIR.parent / "include" / "minimax_moe.h"

MMRS_OK, MMRS_ERR_ARG, MMRS_ERR_UNSUPPORTED, MMRS_ERR_LAUNCH, MMRS_ERR_TIMEOUT, MMRS_ERR_ALLOC = range(6)
MMRS_ERR_SCRATCH_LIMIT = 6
MMRS_ERR_NONFINITE = 7
Q8_0, Q4K, Q2K, Q3K, Q5K, Q6K = 0, 1, 2, 3, 4, 5
ERROR_NAMES = {0: "ok", 1: "invalid argument", 2: "unsupported", 3: "launch failure", 4: "device wait timed out",
               5: "allocation failure", 6: "problem exceeds the fixed scratch", 7: "non-finite value"}


class MoeError(RuntimeError):
    def __init__(self, code: int, what: str):
        super().__init__(f"{what}: {ERROR_NAMES.get(code, code)} ({code})")
        self.code = code


class MmrsMoeWeights(C.Structure):
    _fields_ = [("router", C.c_void_p), ("bias", C.c_void_p), ("gate", C.c_void_p), ("up", C.c_void_p),
                ("down", C.c_void_p), ("gate_up_type", C.c_int), ("down_type", C.c_int),
                ("num_experts", C.c_int), ("topk", C.c_int), ("hidden", C.c_int), ("inter", C.c_int)]


class MmrsPeerGroup(C.Structure):
    _fields_ = [("world", C.c_int), ("rank", C.c_int), ("mine", C.c_void_p), ("peers", C.c_void_p * 8),
                ("ar_capacity", C.c_size_t), ("expert_parallel", C.c_int)]


_VP, _I, _U32, _U64, _I64, _F = C.c_void_p, C.c_int, C.c_uint32, C.c_uint64, C.c_int64, C.c_float
_SZ = C.c_size_t


class MmrsLmHead(C.Structure):
    _fields_ = [("weight", C.c_void_p), ("norm_weight", C.c_void_p), ("vocab", C.c_int), ("hidden", C.c_int),
                ("eps", C.c_float)]


class MmrsSamplingParams(C.Structure):
    """include/minimax_sample.h: SamplingParams (src/sampling.rs:13-17)."""
    _fields_ = [("temperature", C.c_double), ("top_p", C.c_double), ("top_k", C.c_int)]


class MmrsAttnWeights(C.Structure):
    """include/minimax_attn.h: MmrsAttnWeights."""
    _fields_ = [("wq", C.c_void_p), ("wk", C.c_void_p), ("wv", C.c_void_p), ("wo", C.c_void_p),
                ("q_norm", C.c_void_p), ("k_norm", C.c_void_p), ("rope_cos", C.c_void_p), ("rope_sin", C.c_void_p),
                ("hidden", C.c_int), ("query_heads", C.c_int), ("kv_heads", C.c_int), ("rope_dim", C.c_int),
                ("max_positions", C.c_int), ("eps", C.c_float)]

# name -> (restype, argtypes)
PROTOTYPES = {
    "minimax_moe_decode_topk": (None, [_VP] * 7),
    "moe_gemm_gguf_decode_silu": (None, [_VP] * 8 + [_I] * 6 + [_VP]),
    "moe_gemm_gguf": (None, [_VP] * 6 + [_I] * 6 + [_VP]),
    "moe_gemm_mmq_gguf": (None, [_VP] * 6 + [_I] * 6 + [_VP]),
    "moe_sort_routes": (None, [_VP] * 3 + [_I] * 2 + [_VP]),
    "mmrs_last_error": (_I, []),
    # decode attention (include/minimax_attn.h)
    "launch_mmvq_gguf_quantize_q8_1_f32": (None, [_VP, _VP, _I, _I, _I, _VP]),
    "launch_mmvq_gguf_q8_0_f32_plain": (None, [_VP] * 3 + [_I] * 5 + [_VP]),
    "launch_mmvq_gguf_qkv_q8_0_f32": (None, [_VP] * 6 + [_I] * 5 + [_VP]),
    "launch_mmvq_gguf_qkv_q8_0_f32_rmsnorm_f16": (None, [_VP] * 9 + [_I] * 5 + [_F, _VP]),
    "launch_partial_rope_f16": (None, [_VP] * 5 + [_I] * 5 + [_VP]),
    "launch_qkv_tp_sumsq_f32": (None, [_VP] * 3 + [_I] * 2 + [_VP]),
    "launch_qkv_tp_rmsnorm_rope_f16": (None, [_VP] * 9 + [_I] * 8 + [_F, _VP]),
    "launch_gqa_decode_mma_f16_128": (None, [_VP] * 5 + [_I] * 7 + [_F, _I, _VP]),
    "mmrs_attn_workspace_bytes": (_SZ, [C.POINTER(MmrsAttnWeights)]),
    "mmrs_attn_workspace_status": (_I, [_VP]),
    "launch_mmvq_gguf_q6_k_f32_plain": (None, [_VP] * 3 + [_I] * 5 + [_VP]),
    "mmrs_lm_head_workspace_bytes": (_SZ, [C.POINTER(MmrsLmHead)]),
    "mmrs_lm_head_workspace_status": (_I, [_VP]),
    "mmrs_lm_head_forward": (_I, [C.POINTER(MmrsLmHead), _VP, _VP, _VP, _VP, _SZ, _VP]),
    "mmrs_rmsnorm_f32": (_I, [_VP, _VP, _VP, _I, _I, _F, _VP]),
    # token sampling (include/minimax_sample.h)
    "mmrs_sample_workspace_bytes": (_SZ, [_I]),
    "mmrs_sample_workspace_status": (_I, [_VP]),
    "mmrs_sample_token": (_I, [_VP, _I, C.POINTER(MmrsSamplingParams), C.c_double, _VP, _VP, _SZ, _VP]),
    "mmrs_token_logprob": (_I, [_VP, _I, _I, _VP, _VP, _SZ, _VP]),
    "mmrs_attn_decode_forward": (_I, [C.POINTER(MmrsAttnWeights), _VP, _VP, _I, _VP, _VP, _VP, _VP, _SZ, _VP]),
    "launch_tp2_peer_all_reduce_f32": (None, [_VP] * 8 + [C.c_uint, _I, _F, _VP]),
    "launch_tp2_peer_broadcast_f32": (None, [_VP] * 4 + [C.c_uint, _I, _I, _VP]),
    "mmrs_xch_bytes": (_SZ, [_SZ]),
    "mmrs_peer_alloc": (_I, [_SZ, C.POINTER(C.c_void_p)]),
    "mmrs_peer_free": (_I, [_VP]),
    "mmrs_ipc_handle": (_I, [_VP, C.POINTER(C.c_uint8)]),
    "mmrs_ipc_open": (_I, [C.POINTER(C.c_uint8), C.POINTER(C.c_void_p)]),
    "mmrs_ipc_close": (_I, [_VP]),
    "mmrs_peer_enable": (_I, [_I]),
    "mmrs_xch_ar_buffer": (_VP, [C.POINTER(MmrsPeerGroup), _U32]),
    "mmrs_peer_all_reduce": (_I, [C.POINTER(MmrsPeerGroup), _VP, _VP, _SZ, _U32, _VP]),
    "mmrs_peer_status": (_I, [C.POINTER(MmrsPeerGroup), _VP]),
    "mmrs_moe_block_forward_group": (_I, [C.POINTER(MmrsMoeWeights), C.POINTER(MmrsPeerGroup), _VP, _VP, _VP, _I,
                                          _VP, _VP, _VP, _SZ, _U32, _VP]),
    "mmrs_moe_block_forward_group_host": (_I, [C.POINTER(MmrsMoeWeights), C.POINTER(MmrsPeerGroup), _VP, _VP, _VP,
                                               _I, _VP, _VP, _VP, _VP, _VP, _SZ, _U32, _VP]),
    "mmrs_moe_workspace_bytes": (_SZ, [C.POINTER(MmrsMoeWeights), _I]),
    "mmrs_moe_workspace_zero_bytes": (_SZ, [C.POINTER(MmrsMoeWeights)]),
    "mmrs_int8_tensor_peak": (_I, [_I, _I, C.POINTER(C.c_double), _VP]),
    "mmrs_moe_block_forward": (_I, [C.POINTER(MmrsMoeWeights), _VP, _VP, _VP, _I, _VP, _VP, _VP, _SZ, _VP]),
    "mmrs_moe_block_forward_host": (_I, [C.POINTER(MmrsMoeWeights), _VP, _VP, _VP, _I, _VP, _VP, _VP, _VP, _VP, _SZ,
                                         _VP]),
    "mmrs_moe_workspace_status": (_I, [_VP, _VP]),
    "mmrs_moe_block_decode_static": (_I, [C.POINTER(MmrsMoeWeights), _VP, _VP, _VP, _VP, _VP, _VP]),
    "mmrs_moe_static_status": (_I, [_VP]),
    "mmrs_moe_workspace_trace": (_I, [_VP, _VP, _I, _VP]),
    "mmrs_synth_normal_f32": (_I, [_VP, _I64, _U64, _U32, _F, _I, _VP]),
    "mmrs_synth_kquant": (_I, [_VP, _I, _U64, _U32] + [_I] * 7 + [_VP]),
}

_lib = None


def lib() -> C.CDLL:
    """Loads the CUDA library (raises if it has not been built: there is no fallback)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: run `python minimax-rs_b200/build.py` "
                               "(the MoE path has no CPU fallback)")
        l = C.CDLL(str(LIB_PATH))
        for name, (res, args) in PROTOTYPES.items():
            f = getattr(l, name)
            f.restype = res
            f.argtypes = args
        _lib = l
    return _lib


def check(code: int, what: str) -> None:
    if code != MMRS_OK:
        raise MoeError(code, what)


def last_error() -> int:
    return lib().mmrs_last_error()


# ---------------------------------------------------------------------------------------------
# torch helpers
# ---------------------------------------------------------------------------------------------
def _ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(stream=None) -> int:
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def row_bytes(gguf_type: int, k: int) -> int:
    return (k // 256) * (176 if gguf_type == Q5K else 144)


class MoeLayer:
    """Device-resident weights of one MoE layer + the C struct that points at them."""

    def __init__(self, router, bias, gate, up, down, gate_up_type: int, down_type: int, topk: int = 8):
        self.router, self.bias, self.gate, self.up, self.down = router, bias, gate, up, down
        self.num_experts, self.hidden = router.shape
        self.inter = gate.numel() // (self.num_experts * row_bytes(gate_up_type, self.hidden))
        self.c = MmrsMoeWeights(router.data_ptr(), bias.data_ptr(), gate.data_ptr(), up.data_ptr(),
                                down.data_ptr(), gate_up_type, down_type, self.num_experts, topk,
                                self.hidden, self.inter)
        self.topk = topk
        self._ws = None

    def workspace(self, max_tokens: int):
        import torch
        nbytes = lib().mmrs_moe_workspace_bytes(C.byref(self.c), max_tokens)
        if self._ws is None or self._ws.numel() < nbytes:
            self._ws = torch.zeros(nbytes, dtype=torch.uint8, device=self.router.device)
        return self._ws

    def forward(self, x, residual=None, y=None, topk_ids=None, topk_w=None, stream=None):
        """y = MoE(x) (+ residual); x [T, hidden] f32 CUDA tensor."""
        import torch
        T = x.shape[0]
        if y is None:
            y = torch.empty_like(x)
        ws = self.workspace(T)
        rc = lib().mmrs_moe_block_forward(C.byref(self.c), x.data_ptr(), _ptr(residual), y.data_ptr(), T,
                                          _ptr(topk_ids), _ptr(topk_w), ws.data_ptr(), ws.numel(), _stream(stream))
        check(rc, "mmrs_moe_block_forward")
        return y

    def forward_host(self, x_host, y_host, x_dev, y_dev, residual=None, topk_ids=None, topk_w=None, stream=None):
        """y_host = MoE(x_host) (+ residual) in one library call: the copy of x_host [T, hidden]
        (pinned host memory) into x_dev, the block into y_dev and the copy back into y_host are
        enqueued on `stream`; residual / topk_* are CUDA tensors as in forward()."""
        T = x_host.shape[0]
        ws = self.workspace(T)
        rc = lib().mmrs_moe_block_forward_host(C.byref(self.c), x_host.data_ptr(), _ptr(residual), y_host.data_ptr(),
                                               T, x_dev.data_ptr(), y_dev.data_ptr(), _ptr(topk_ids), _ptr(topk_w),
                                               ws.data_ptr(), ws.numel(), _stream(stream))
        check(rc, "mmrs_moe_block_forward_host")
        return y_host

    def trace(self, stream=None):
        """Per-CTA phase timestamps (ns) of the last single-token launch: array [256, 32]."""
        import numpy as np
        out = np.zeros(256 * 32, dtype=np.uint64)
        n = lib().mmrs_moe_workspace_trace(self._ws.data_ptr(), out.ctypes.data, out.size, _stream(stream))
        if n < 0:
            raise MoeError(-n, "mmrs_moe_workspace_trace")
        return out.reshape(256, 32)

    def status(self, stream=None) -> int:
        return lib().mmrs_moe_workspace_status(self._ws.data_ptr(), _stream(stream)) if self._ws is not None else 0


def moe_gemm(inp, weights, sorted_token_ids, expert_ids, topk_weights, out, num_experts: int, topk: int,
             size_n: int, size_k: int, gguf_type: int, mmq: bool = False, stream=None):
    """moe_gemm_gguf / moe_gemm_mmq_gguf through the reference ABI; raises on a recorded error."""
    fn = lib().moe_gemm_mmq_gguf if mmq else lib().moe_gemm_gguf
    fn(inp.data_ptr(), weights.data_ptr(), sorted_token_ids.data_ptr(), expert_ids.data_ptr(), _ptr(topk_weights),
       out.data_ptr(), num_experts, topk, sorted_token_ids.numel(), size_n, size_k, gguf_type, _stream(stream))
    check(last_error(), "moe_gemm_mmq_gguf" if mmq else "moe_gemm_gguf")
    return out


def sort_routes(expert_ids, end_bit: int, stream=None):
    """moe_sort_routes: stable sort of u32 keys on bits [0, end_bit) -> (sorted keys, positions)."""
    import torch
    n = expert_ids.numel()
    keys = torch.empty(n, dtype=torch.int32, device=expert_ids.device)
    routes = torch.empty(n, dtype=torch.int32, device=expert_ids.device)
    lib().moe_sort_routes(expert_ids.data_ptr(), keys.data_ptr(), routes.data_ptr(), n, end_bit, _stream(stream))
    check(last_error(), "moe_sort_routes")
    return keys, routes


def int8_tensor_peak(chunks: int = 4096, reps: int = 5, stream=None) -> float:
    """Measured dense int8 tensor-core throughput of the current device, TOPS (mmrs_int8_tensor_peak)."""
    out = C.c_double(0.0)
    check(lib().mmrs_int8_tensor_peak(chunks, reps, C.byref(out), _stream(stream)), "mmrs_int8_tensor_peak")
    return out.value


def synth_normal(t, seed: int, stream_id: int, scale: float = 1.0, bf16: bool = False, stream=None):
    check(lib().mmrs_synth_normal_f32(t.data_ptr(), t.numel(), seed, stream_id, scale, int(bf16), _stream(stream)),
          "mmrs_synth_normal_f32")
    return t


def synth_kquant(t, gguf_type: int, seed: int, stream_id: int, experts: int, rows: int, k: int,
                 row0: int = 0, nrows: int | None = None, kblk0: int = 0, nkblk: int | None = None, stream=None):
    nrows = rows - row0 if nrows is None else nrows
    nkblk = k // 256 - kblk0 if nkblk is None else nkblk
    check(lib().mmrs_synth_kquant(t.data_ptr(), gguf_type, seed, stream_id, experts, rows, k, row0, nrows, kblk0,
                                  nkblk, _stream(stream)), "mmrs_synth_kquant")
    return t


class AttnLayer:
    """Single-token attention half of a layer (Attention::forward, src/model.rs:79-162, T = 1):
    device-resident Q8_0 weights, RMSNorm weights, rotary tables and the f16 KV cache
    [kv_heads][max_positions][128], with the C struct that points at them."""

    def __init__(self, wq, wk, wv, wo, q_norm, k_norm, rope_cos, rope_sin, hidden: int, query_heads: int = 48,
                 kv_heads: int = 8, rope_dim: int = 64, eps: float = 1e-6):
        import torch
        self.t = (wq, wk, wv, wo, q_norm, k_norm, rope_cos, rope_sin)
        self.max_positions = rope_cos.shape[0]
        self.c = MmrsAttnWeights(wq.data_ptr(), wk.data_ptr(), wv.data_ptr(), wo.data_ptr(), q_norm.data_ptr(),
                                 k_norm.data_ptr(), rope_cos.data_ptr(), rope_sin.data_ptr(), hidden, query_heads,
                                 kv_heads, rope_dim, self.max_positions, eps)
        dev = wq.device
        self.k_cache = torch.zeros(kv_heads, self.max_positions, 128, dtype=torch.float16, device=dev)
        self.v_cache = torch.zeros_like(self.k_cache)
        self.ws = torch.zeros(lib().mmrs_attn_workspace_bytes(C.byref(self.c)), dtype=torch.uint8, device=dev)
        if self.ws.numel() == 0:
            raise MoeError(MMRS_ERR_UNSUPPORTED, "mmrs_attn_workspace_bytes")

    def status(self) -> int:
        """MMRS_OK, or MMRS_ERR_TIMEOUT when a bounded wait in the attention kernel expired."""
        return lib().mmrs_attn_workspace_status(self.ws.data_ptr())

    def forward(self, x, position: int, residual=None, y=None, stream=None):
        """y [hidden] f32 = Wo . attention(x) (+ residual); appends the token's K / V at `position`."""
        import torch
        if y is None:
            y = torch.empty_like(x)
        rc = lib().mmrs_attn_decode_forward(C.byref(self.c), x.data_ptr(), _ptr(residual), position,
                                            self.k_cache.data_ptr(), self.v_cache.data_ptr(), y.data_ptr(),
                                            self.ws.data_ptr(), self.ws.numel(), _stream(stream))
        check(rc, "mmrs_attn_decode_forward")
        return y


class LmHead:
    """Output projection of a decode step (TensorParallelModel::logits, src/tensor_parallel_model.rs:871-880,
    and greedy sampling, src/sampling.rs:84-88): device-resident Q6_K `output.weight` [vocab][hidden]
    and `output_norm.weight` (or None), with the C struct that points at them."""

    def __init__(self, weight, norm_weight, vocab: int, hidden: int, eps: float = 1e-6):
        import torch
        self.t = (weight, norm_weight)
        self.c = MmrsLmHead(weight.data_ptr(), _ptr(norm_weight), vocab, hidden, eps)
        n = lib().mmrs_lm_head_workspace_bytes(C.byref(self.c))
        if n == 0:
            raise MoeError(MMRS_ERR_UNSUPPORTED, "mmrs_lm_head_workspace_bytes")
        self.ws = torch.zeros(n, dtype=torch.uint8, device=weight.device)
        self.logits = torch.empty(vocab, dtype=torch.float32, device=weight.device)
        self.token = torch.zeros(1, dtype=torch.int32, device=weight.device)

    def status(self) -> int:
        return lib().mmrs_lm_head_workspace_status(self.ws.data_ptr())

    def forward(self, x, stream=None):
        """(logits [vocab] f32, token [1] int32) for the final hidden state x [hidden] f32."""
        rc = lib().mmrs_lm_head_forward(C.byref(self.c), x.data_ptr(), self.logits.data_ptr(), self.token.data_ptr(),
                                        self.ws.data_ptr(), self.ws.numel(), _stream(stream))
        check(rc, "mmrs_lm_head_forward")
        return self.logits, self.token


DEFAULT_TEMPERATURE, DEFAULT_TOP_P, DEFAULT_TOP_K = 1.0, 0.95, 40  # src/sampling.rs:6-8


class Sampler:
    """TokenSampler (src/sampling.rs:43-150) over device logits: greedy at temperature 0, else top-k,
    top-p and temperature sampling, the choice made on the device (mmrs_sample_token).  The uniform
    draw is the caller's: `sample(logits, u)` takes it, or draws it from this sampler's own
    generator (numpy PCG64 seeded with `seed`; the reference draws from a per-request StdRng) only
    when the temperature is positive, as the reference draws only then."""

    def __init__(self, vocab: int, device, temperature: float = DEFAULT_TEMPERATURE, top_p: float = DEFAULT_TOP_P,
                 top_k: int = DEFAULT_TOP_K, seed: int = 0):
        import math

        import numpy as np
        import torch
        # SamplingParams::validate (src/sampling.rs:31-39)
        if not math.isfinite(temperature) or temperature < 0.0:
            raise MoeError(MMRS_ERR_ARG, "temperature must be a finite number greater than or equal to 0")
        if not math.isfinite(top_p) or not 0.0 <= top_p <= 1.0:
            raise MoeError(MMRS_ERR_ARG, "top_p must be a finite number between 0 and 1")
        self.params = MmrsSamplingParams(float(temperature), float(top_p), int(top_k))
        self.vocab = vocab
        n = lib().mmrs_sample_workspace_bytes(vocab)
        if n == 0:
            raise MoeError(MMRS_ERR_ARG, "mmrs_sample_workspace_bytes")
        self.ws = torch.zeros(n, dtype=torch.uint8, device=device)
        self.token = torch.full((1,), -1, dtype=torch.int32, device=device)
        self.logprob = torch.zeros(1, dtype=torch.float32, device=device)
        self.rng = np.random.default_rng(seed)

    def status(self) -> int:
        """Outcome of the last completed call (synchronous)."""
        return lib().mmrs_sample_workspace_status(self.ws.data_ptr())

    def sample(self, logits, u: float | None = None, stream=None):
        """token [1] int32 on the device (-1 when status() is not MMRS_OK) for logits [vocab] f32."""
        if u is None:
            u = float(self.rng.random()) if self.params.temperature > 0.0 else 0.0
        rc = lib().mmrs_sample_token(logits.data_ptr(), self.vocab, C.byref(self.params), float(u),
                                     self.token.data_ptr(), self.ws.data_ptr(), self.ws.numel(), _stream(stream))
        check(rc, "mmrs_sample_token")
        return self.token

    def token_logprob(self, logits, token_id: int, stream=None):
        """ln softmax(logits)[token_id] as a [1] f32 device tensor (token_logprob, src/sampling.rs:60-75)."""
        rc = lib().mmrs_token_logprob(logits.data_ptr(), self.vocab, int(token_id), self.logprob.data_ptr(),
                                      self.ws.data_ptr(), self.ws.numel(), _stream(stream))
        check(rc, "mmrs_token_logprob")
        return self.logprob


def rmsnorm(x, weight, y=None, eps: float = 1e-6, stream=None):
    """y = x / sqrt(mean(x^2) + eps) * weight over the last dimension (CUDA f32 tensors)."""
    import torch
    if y is None:
        y = torch.empty_like(x)
    n = x.shape[-1]
    check(lib().mmrs_rmsnorm_f32(x.data_ptr(), weight.data_ptr(), y.data_ptr(), n, x.numel() // n, eps,
                                 _stream(stream)), "mmrs_rmsnorm_f32")
    return y
