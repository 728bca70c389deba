"""ctypes wrapper of the CPU oracle (oracle/moe_oracle.c) — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm may import this
module.  The product path (minimax-rs_b200) never does.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"

Q4K, Q5K = 1, 4
BLOCK_BYTES = {Q4K: 144, Q5K: 176}


def build() -> Path:
    src = [HERE / n for n in ("moe_oracle.c", "attn_oracle.c", "lmhead_oracle.c", "sample_oracle.c", "moe_oracle.h",
                              "Makefile")]
    if not LIB_PATH.exists() or any(s.stat().st_mtime > LIB_PATH.stat().st_mtime for s in src):
        subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


class OrcMoeWeights(C.Structure):
    _fields_ = [("router", C.c_void_p), ("bias", C.c_void_p), ("gate", C.c_void_p), ("up", C.c_void_p),
                ("down", C.c_void_p), ("gate_up_type", C.c_int), ("down_type", C.c_int),
                ("num_experts", C.c_int), ("topk", C.c_int), ("hidden", C.c_int), ("inter", C.c_int)]


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        build()
        _lib = C.CDLL(str(LIB_PATH))
        _lib.orc_half_to_float.restype = C.c_float
        _lib.orc_half_to_float.argtypes = [C.c_uint16]
        _lib.orc_float_to_half.restype = C.c_uint16
        _lib.orc_float_to_half.argtypes = [C.c_float]
        _lib.orc_dot_q4k_q81.restype = C.c_float
        _lib.orc_dot_q5k_q81.restype = C.c_float
        _lib.orc_dot_kq_mmq.restype = C.c_float
        _lib.orc_num_threads.restype = C.c_int
        _lib.orc_argmax_f32.restype = C.c_int
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def num_threads() -> int:
    return lib().orc_num_threads()


def set_threads(n: int = 0) -> int:
    """OpenMP team size of later calls (0: every hardware thread); returns the size now in force."""
    lib().orc_set_threads(C.c_int(n))
    return num_threads()


def dequant(gguf_type: int, blocks: np.ndarray, fused: bool = True) -> np.ndarray:
    b = _c(blocks, np.uint8).reshape(-1)
    n = b.size // BLOCK_BYTES[gguf_type]
    out = np.empty(n * 256, dtype=np.float32)
    f = lib().orc_dequant_q4k if gguf_type == Q4K else lib().orc_dequant_q5k
    f(_p(b), C.c_int64(n), _p(out), C.c_int(int(fused)))
    return out


def quantize_q8_1(x: np.ndarray, kpad: int | None = None) -> np.ndarray:
    x = _c(x, np.float32)
    rows, k = x.reshape(-1, x.shape[-1]).shape
    kpad = kpad or (k + 511) // 512 * 512
    out = np.empty((rows, kpad // 32, 36), dtype=np.uint8)
    lib().orc_quantize_q8_1(_p(x), C.c_int(rows), C.c_int(k), C.c_int(kpad), _p(out))
    return out


def quantize_q8_1_mmq(x: np.ndarray, src_rows=None, rows: int | None = None, kpad: int | None = None):
    x = _c(x, np.float32)
    k = x.shape[-1]
    kpad = kpad or (k + 511) // 512 * 512
    src = None if src_rows is None else _c(src_rows, np.int32)
    rows = rows if rows is not None else (len(src) if src is not None else x.reshape(-1, k).shape[0])
    q = np.empty((rows, kpad), dtype=np.int8)
    d = np.empty((rows, kpad // 32), dtype=np.uint16)
    s = np.empty((rows, kpad // 32), dtype=np.uint16)
    lib().orc_quantize_q8_1_mmq(_p(x), _p(src), C.c_int(rows), C.c_int(k), C.c_int(kpad), _p(q), _p(d), _p(s))
    return q, d, s


def router_logits(x: np.ndarray, wr: np.ndarray) -> np.ndarray:
    x = _c(x, np.float32)
    wr = _c(wr, np.float32)
    T, K = x.reshape(-1, x.shape[-1]).shape
    E = wr.shape[0]
    out = np.empty((T, E), dtype=np.float32)
    lib().orc_router_logits(_p(x), _p(wr), C.c_int(T), C.c_int(E), C.c_int(K), _p(out))
    return out


def route_topk(logits: np.ndarray, bias: np.ndarray, topk: int = 8):
    lg = _c(logits, np.float32)
    T, E = lg.shape
    ids = np.empty((T, topk), dtype=np.uint32)
    w = np.empty((T, topk), dtype=np.float32)
    lib().orc_route_topk(_p(lg), _p(_c(bias, np.float32)), C.c_int(T), C.c_int(E), C.c_int(topk), _p(ids), _p(w))
    return ids, w


def decode_topk(logits: np.ndarray, bias: np.ndarray):
    lg = _c(logits, np.float32).reshape(256)
    ids = np.empty(8, np.uint32)
    w = np.empty(8, np.float32)
    e = np.empty(8, np.uint32)
    r = np.empty(8, np.uint32)
    lib().orc_decode_topk(_p(lg), _p(_c(bias, np.float32)), _p(ids), _p(w), _p(e), _p(r))
    return ids, w, e, r


def sort_routes(expert_ids: np.ndarray):
    e = _c(expert_ids, np.uint32).reshape(-1)
    se = np.empty_like(e)
    sr = np.empty_like(e)
    lib().orc_sort_routes(_p(e), C.c_int(e.size), _p(se), _p(sr))
    return se, sr


def moe_gemm_gguf(inp, weights, sorted_token_ids, expert_ids, topk_weights, num_experts, topk, size_m, size_n,
                  size_k, gguf_type, mmq: bool = False):
    out = np.zeros((size_m, size_n), dtype=np.float32)
    f = lib().orc_moe_gemm_mmq if mmq else lib().orc_moe_gemm_gguf
    tw = None if topk_weights is None else _c(topk_weights, np.float32)
    f(_p(_c(inp, np.float32)), _p(_c(weights, np.uint8)), _p(_c(sorted_token_ids, np.int32)),
      _p(_c(expert_ids, np.int32)), _p(tw), _p(out), C.c_int(num_experts), C.c_int(topk), C.c_int(size_m),
      C.c_int(size_n), C.c_int(size_k), C.c_int(gguf_type))
    return out


def moe_decode_silu(inp, gate, up, down, sorted_token_ids, expert_ids, topk_weights, num_experts, hidden, inter,
                    gate_up_type, down_type):
    out = np.zeros(hidden, dtype=np.float32)
    lib().orc_moe_decode_silu(_p(_c(inp, np.float32)), _p(_c(gate, np.uint8)), _p(_c(up, np.uint8)),
                              _p(_c(down, np.uint8)), _p(_c(sorted_token_ids, np.int32)),
                              _p(_c(expert_ids, np.int32)), _p(_c(topk_weights, np.float32)), _p(out),
                              C.c_int(num_experts), C.c_int(8), C.c_int(hidden), C.c_int(inter),
                              C.c_int(gate_up_type), C.c_int(down_type))
    return out


def moe_block(router, bias, gate, up, down, gate_up_type, down_type, x, residual=None, topk: int = 8,
              mmq_min_tokens: int = 32):
    """FusedMoeGGUF::forward (+ residual) on the CPU.  Returns (y, topk_ids, topk_w)."""
    router = _c(router, np.float32)
    bias = _c(bias, np.float32)
    gate, up, down = _c(gate, np.uint8), _c(up, np.uint8), _c(down, np.uint8)
    E, H = router.shape
    inter = gate.size // (E * (H // 256) * BLOCK_BYTES[gate_up_type])
    w = OrcMoeWeights(_p(router).value, _p(bias).value, _p(gate).value, _p(up).value, _p(down).value,
                      gate_up_type, down_type, E, topk, H, inter)
    x = _c(x, np.float32).reshape(-1, H)
    T = x.shape[0]
    y = np.empty((T, H), dtype=np.float32)
    ids = np.empty((T, topk), dtype=np.uint32)
    tw = np.empty((T, topk), dtype=np.float32)
    res = None if residual is None else _c(residual, np.float32).reshape(T, H)
    lib().orc_moe_block(C.byref(w), _p(x), _p(res), C.c_int(T), C.c_int(mmq_min_tokens), _p(y), _p(ids), _p(tw))
    return y, ids, tw


# ---- decode attention (attn_oracle.c) ----------------------------------------------------
def q8_0_matvec(w: np.ndarray, rows: int, k: int, x: np.ndarray) -> np.ndarray:
    """y = W x for a Q8_0 matrix (rows x k/32 blocks of 34 bytes), x quantised to Q8_1."""
    w, x = _c(w, np.uint8), _c(x, np.float32)
    y = np.zeros(rows, dtype=np.float32)
    lib().orc_q8_0_matvec(_p(w), C.c_int(rows), C.c_int(k), _p(x), _p(y))
    return y


def q6k_matvec(w: np.ndarray, rows: int, k: int, x: np.ndarray) -> np.ndarray:
    """y = W x for a Q6_K matrix (rows x k/256 blocks of 210 bytes), x quantised to Q8_1
    (lmhead_oracle.c; exact up to the final rounding)."""
    w, x = _c(w, np.uint8), _c(x, np.float32)
    y = np.zeros(rows, dtype=np.float32)
    lib().orc_q6k_matvec(_p(w), C.c_int(rows), C.c_int(k), _p(x), _p(y))
    return y


def q6k_dequant_row(row: np.ndarray, k: int) -> np.ndarray:
    out = np.zeros(k, dtype=np.float32)
    lib().orc_q6k_dequant_row(_p(_c(row, np.uint8)), C.c_int(k), _p(out))
    return out


def argmax_f32(v: np.ndarray) -> int:
    """First index of the maximum (the reference's greedy choice)."""
    v = _c(v, np.float32)
    return int(lib().orc_argmax_f32(_p(v), C.c_int(v.size)))


def sample_token(logits: np.ndarray, temperature: float, top_p: float, top_k: int, u: float):
    """(status, token, margin) of TokenSampler::sample for the draw u (sample_oracle.c); status 0,
    1 (invalid parameters) or 7 (non-finite logits)."""
    v = _c(logits, np.float32)
    tok = C.c_int32(-1)
    margin = C.c_double(0.0)
    st = lib().orc_sample_token(_p(v), C.c_int(v.size), C.c_double(temperature), C.c_double(top_p), C.c_int(top_k),
                                C.c_double(u), C.byref(tok), C.byref(margin))
    return int(st), int(tok.value), float(margin.value)


def token_logprob(logits: np.ndarray, token_id: int):
    """(status, ln softmax(logits)[token_id]) (sample_oracle.c); status 0, 1 or 7."""
    v = _c(logits, np.float32)
    out = C.c_float(0.0)
    st = lib().orc_token_logprob(_p(v), C.c_int(v.size), C.c_int(token_id), C.byref(out))
    return int(st), float(out.value)


def qkv_rmsnorm_f16(proj, q_alpha, k_alpha, q_rows: int, k_rows: int, v_rows: int, eps: float = 1e-6):
    """f16 bits (uint16) of [RMSNorm(q) * q_alpha | RMSNorm(k) * k_alpha | v]."""
    proj, qa, ka = _c(proj, np.float32), _c(q_alpha, np.float32), _c(k_alpha, np.float32)
    out = np.zeros(q_rows + k_rows + v_rows, dtype=np.uint16)
    lib().orc_qkv_rmsnorm_f16(_p(proj), _p(qa), _p(ka), C.c_int(q_rows), C.c_int(k_rows), C.c_int(v_rows),
                              C.c_float(eps), _p(out))
    return out


def partial_rope_f16(q, k, cos, sin, head_dim: int, rope_dim: int, position: int):
    """f16 bits of [rotated q | rotated k]; q / k given as float16 or uint16 bit arrays."""
    q, k = _c(np.asarray(q).view(np.uint16), np.uint16), _c(np.asarray(k).view(np.uint16), np.uint16)
    cos, sin = _c(cos, np.float32), _c(sin, np.float32)
    out = np.zeros(q.size + k.size, dtype=np.uint16)
    lib().orc_partial_rope_f16(_p(q), _p(k), _p(cos), _p(sin), C.c_int(q.size), C.c_int(k.size), C.c_int(head_dim),
                               C.c_int(rope_dim), C.c_int(position), _p(out))
    return out


def tp_qk_sumsq(q: np.ndarray, k: np.ndarray) -> np.ndarray:
    """[sum q^2, sum k^2] of one tensor-parallel rank's projection (launch_qkv_tp_sumsq_f32,
    mmvq_gguf.cu:970-990), accumulated in double."""
    q, k = np.asarray(q, np.float64), np.asarray(k, np.float64)
    return np.array([np.dot(q, q), np.dot(k, k)])


def tp_qk_rmsnorm_rope_f16(q, k, v, global_stats, q_alpha, k_alpha, cos, sin, q_full: int, k_full: int,
                           head_dim: int, rope_dim: int, position: int, eps: float = 1e-6) -> np.ndarray:
    """f16 bits of [rope(q * s_q * q_alpha) | rope(k * s_k * k_alpha) | v] for one TP rank
    (launch_qkv_tp_rmsnorm_rope_f16, mmvq_gguf.cu:995-1034): s = 1 / sqrt(global / full + eps) with
    the global (all-rank) sums, computed here in double and rounded to f32 (the kernel's rsqrtf is
    within 2 ulp of it); the products in f32, rounded to half; the rotation with the reference's
    half arithmetic (partial_rope_f16); v rounded to half."""
    g = np.asarray(global_stats, np.float32)
    sq = np.float32(1.0 / np.sqrt(np.float64(np.float32(g[0] / np.float32(q_full)) + np.float32(eps))))
    sk = np.float32(1.0 / np.sqrt(np.float64(np.float32(g[1] / np.float32(k_full)) + np.float32(eps))))
    qh = ((sq * np.asarray(q, np.float32)) * np.asarray(q_alpha, np.float32)).astype(np.float16)
    kh = ((sk * np.asarray(k, np.float32)) * np.asarray(k_alpha, np.float32)).astype(np.float16)
    rot = partial_rope_f16(qh, kh, cos, sin, head_dim, rope_dim, position)
    return np.concatenate([rot, np.asarray(v, np.float32).astype(np.float16).view(np.uint16)])


def gqa_decode_f16(q, k, v, seq_len: int, q_heads: int, kv_heads: int, head_dim: int, kv_head_stride: int,
                   scale: float):
    """f16 bits [q_heads * head_dim] of softmax(scale q.k) v over positions [0, seq_len)."""
    q = _c(np.asarray(q).view(np.uint16), np.uint16)
    k = _c(np.asarray(k).view(np.uint16), np.uint16)
    v = _c(np.asarray(v).view(np.uint16), np.uint16)
    out = np.zeros(q_heads * head_dim, dtype=np.uint16)
    lib().orc_gqa_decode_f16(_p(q), _p(k), _p(v), C.c_int(seq_len), C.c_int(q_heads), C.c_int(kv_heads),
                             C.c_int(head_dim), C.c_int64(kv_head_stride), C.c_float(scale), _p(out))
    return out
