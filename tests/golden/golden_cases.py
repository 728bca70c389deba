"""Seeded cases of the reference-kernel golden vectors (tests/golden/ref_kernels.npz).

Shared by make_golden.py (which runs the reference's own kernels on a GPU) and by the parity tests
(which regenerate the same inputs and compare the oracle / the CUDA path with the stored outputs).
Every input is a pure function of fixed seeds through minimax-rs_b200/synth.py.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
import __graft_entry__ as _ge  # noqa: E402

S = _ge.load_synth()
Q4K, Q5K = 1, 4
QUANT_K = (512, 768)


def _perm(seed: int, stream: int, n: int) -> np.ndarray:
    key = S.stream_key(seed, stream)
    return np.argsort(S.rand64(key, np.arange(n, dtype=np.uint64)), kind="stable")


def dequant_blocks(gt: int) -> np.ndarray:
    w = S.kquant(gt, 501, 1 if gt == Q4K else 2, 1, 16, 1024)
    bb = 144 if gt == Q4K else 176
    return w.reshape(-1, bb)  # 64 super-blocks


def quant_input(kx: int) -> np.ndarray:
    x = S.normal_f32(4 * kx, 502, kx, 3.0).reshape(4, kx)
    x[1, 32:64] = 0.0  # an all-zero Q8_1 block
    return x


def mmq_quant_case():
    kx, div = 768, 4  # kx pads to 1024: four all-zero 32-blocks per row
    x = S.normal_f32(6 * kx, 503, 1, 2.0).reshape(6, kx)
    ids = (_perm(503, 2, 24)[:12]).astype(np.int32)  # route ids, source row = id // div
    return x, ids, kx, div


def topk_inputs():
    lg = S.normal_f32(24 * 256, 504, 1, 1.1).reshape(24, 256)
    bias = S.normal_f32(256, 504, 2, 0.01)
    # exact tie between experts 10 and 20 in set 0, both among the selected
    bias[20] = bias[10]
    lg[0, 10] = lg[0, 20] = 6.0
    return lg, bias


DECODE_CASES = (
    dict(name="e16_h512_i256", E=16, H=512, I=256, gu=Q4K, dn=Q5K, seed=601),
    dict(name="e16_h512_i768", E=16, H=512, I=768, gu=Q4K, dn=Q5K, seed=602),
    dict(name="e8_h1024_i256_q4k", E=8, H=1024, I=256, gu=Q4K, dn=Q4K, seed=603),
)


def layer(c):
    st = S.layer_streams(0)
    E, H, I = c["E"], c["H"], c["I"]
    return dict(gate=S.kquant(c["gu"], c["seed"], st["gate"], E, I, H),
                up=S.kquant(c["gu"], c["seed"], st["up"], E, I, H),
                down=S.kquant(c["dn"], c["seed"], st["down"], E, H, I))


def token(c):
    return S.normal_f32(c["H"], c["seed"], S.layer_streams(0)["x"], 1.0, bf16=True)


def decode_routing(c):
    """(route ids, expert ids) pairs in expert order + weights indexed by route."""
    experts = np.sort(_perm(c["seed"], 10, c["E"])[:8]).astype(np.int32)
    routes = _perm(c["seed"], 11, 8).astype(np.int32)
    w = np.abs(S.normal_f32(8, c["seed"], 12, 1.0)) + np.float32(0.05)
    return routes, experts, (w / w.sum()).astype(np.float32)


GEMM_CASES = (
    dict(name="generic_gate_q4k", mmq=False, T=4, E=16, N=128, K=512, type=Q4K, down=False, seed=701),
    dict(name="generic_down_q5k", mmq=False, T=4, E=16, N=512, K=256, type=Q5K, down=True, seed=702),
    dict(name="mmq_gate_q4k", mmq=True, T=40, E=16, N=128, K=512, type=Q4K, down=False, seed=703),
    dict(name="mmq_down_q5k", mmq=True, T=40, E=16, N=512, K=256, type=Q5K, down=True, seed=704),
)
for _c in GEMM_CASES:
    _c["M"] = _c["T"] * 8


def gemm_routing(c):
    """Per token 8 distinct experts; flattened route ids stably sorted by expert."""
    T, E = c["T"], c["E"]
    ids = np.stack([_perm(c["seed"], 100 + t, E)[:8] for t in range(T)]).astype(np.uint32)
    flat = ids.reshape(-1)
    order = np.argsort(flat, kind="stable").astype(np.int32)
    return ids, order, flat[order].astype(np.int32)


def gemm_inputs(c):
    _, sorted_ids, experts = gemm_routing(c)
    rows = c["M"] if c["down"] else c["T"]
    inp = S.normal_f32(rows * c["K"], c["seed"], 1, 30.0 if c["down"] else 1.0).reshape(rows, c["K"])
    w = S.kquant(c["type"], c["seed"], 2, c["E"], c["N"], c["K"])
    tw = None
    if c["down"]:
        tw = (np.abs(S.normal_f32(c["M"], c["seed"], 3, 1.0)) * np.float32(0.2)).astype(np.float32)
    return inp, w, sorted_ids, experts, tw


def sort_input() -> np.ndarray:
    key = S.stream_key(801, 1)
    return (S.rand64(key, np.arange(2048 * 8, dtype=np.uint64)) % np.uint64(256)).astype(np.uint32)


def mmq_layout_to_logical(vy: np.ndarray, rows: int, kpad: int):
    """block_q8_1_mmq buffer (mmq_gguf.cuh:28-54; block index = (k / 128) * rows + row, each
    block = half2 ds4[4] then 128 int8) -> (q [rows][kpad] int8, d, s [rows][kpad/32] half bits)."""
    nb = kpad // 128
    blk = vy.reshape(nb, rows, 144)
    ds = blk[:, :, :16].copy().view(np.uint16).reshape(nb, rows, 4, 2)
    q = blk[:, :, 16:].view(np.int8).transpose(1, 0, 2).reshape(rows, kpad)
    d = ds[..., 0].transpose(1, 0, 2).reshape(rows, nb * 4)
    s = ds[..., 1].transpose(1, 0, 2).reshape(rows, nb * 4)
    return q, d, s


# ------------------------------------------------------------------------------------------
# Decode attention (tests/golden/ref_attn.npz): MiniMax's fixed head geometry (48 query heads,
# 8 KV heads, head dim 128, rotary dims 64, theta 5e6) at the model's hidden size.
# ------------------------------------------------------------------------------------------
ATTN_H, QH, KVH, HD, ROT = 3072, 48, 8, 128, 64
Q_ROWS, K_ROWS, V_ROWS = QH * HD, KVH * HD, KVH * HD
ROPE_POS = (0, 7, 4095)
ROPE_MAX_POS = 4096
KV_CAP = 4096  # cache capacity (positions per KV head)
GQA_CASES = ((1, 1), (129, 4), (1000, 16), (4096, 32))  # (seq_len, num_splits)


def qkv_inputs():
    x = S.normal_f32(ATTN_H, 701, 1, 1.0)
    wq = S.q8_0_blocks(701, 2, Q_ROWS, ATTN_H)
    wk = S.q8_0_blocks(701, 3, K_ROWS, ATTN_H)
    wv = S.q8_0_blocks(701, 4, V_ROWS, ATTN_H)
    qa = (1.0 + S.normal_f32(Q_ROWS, 701, 5, 0.1)).astype(np.float32)
    ka = (1.0 + S.normal_f32(K_ROWS, 701, 6, 0.1)).astype(np.float32)
    return x, wq, wk, wv, qa, ka


def rope_inputs():
    q = S.normal_f16(Q_ROWS, 702, 1, 1.0)
    k = S.normal_f16(K_ROWS, 702, 2, 1.0)
    cos, sin = S.rope_tables(ROPE_MAX_POS, ROT)
    return q, k, cos, sin


def gqa_inputs(seq_len: int):
    """q [48][128] and K / V caches [8][KV_CAP][128] (positions >= seq_len are zero), half."""
    q = S.normal_f16(QH * HD, 703, 1, 1.0).reshape(QH, HD)
    k = np.zeros((KVH, KV_CAP, HD), dtype=np.float16)
    v = np.zeros((KVH, KV_CAP, HD), dtype=np.float16)
    k[:, :seq_len] = S.normal_f16(KVH * KV_CAP * HD, 703, 2, 1.0).reshape(KVH, KV_CAP, HD)[:, :seq_len]
    v[:, :seq_len] = S.normal_f16(KVH * KV_CAP * HD, 703, 3, 1.0).reshape(KVH, KV_CAP, HD)[:, :seq_len]
    return q, k, v


def oproj_inputs():
    a = S.normal_f16(Q_ROWS, 704, 1, 1.0).astype(np.float32)  # attention output, widened
    wo = S.q8_0_blocks(704, 2, ATTN_H, Q_ROWS)
    return a, wo


# ---- LM head (output projection, Q6_K) -------------------------------------------------------
LM_ROWS, LM_K = 4096, 3072  # a slice of the 200064-row vocabulary at the model's hidden size


def lm_inputs():
    """x [3072] f32 (the normed final hidden state) and a Q6_K matrix [4096][12 x 210 B]."""
    x = S.normal_f32(LM_K, 901, 1, 1.0)
    w = S.q6k_blocks(901, 2, LM_ROWS, LM_K)
    return x, w


# ---- tensor-parallel Q/K RMSNorm (TP = 2) ------------------------------------------------------
TP_Q_LOCAL, TP_KV_LOCAL = 24 * 128, 4 * 128  # a rank's 24 query heads and 4 KV heads
TP_Q_FULL, TP_K_FULL = 48 * 128, 8 * 128
TP_POS = (0, 1234)


def tp_qk_inputs(rank: int):
    """A TP = 2 rank's f32 projection q / k / v (the rank's heads), its slices of the Q / K norm
    weights, and the rotary tables.  Rank 1's q is scaled by 3 so the two ranks' sums differ."""
    scale = 1.0 if rank == 0 else 3.0
    q = (S.normal_f32(TP_Q_LOCAL, 911, 1 + 10 * rank, 1.0) * scale).astype(np.float32)
    k = S.normal_f32(TP_KV_LOCAL, 911, 2 + 10 * rank, 2.0)
    v = S.normal_f32(TP_KV_LOCAL, 911, 3 + 10 * rank, 1.0)
    qa_full = (1.0 + S.normal_f32(TP_Q_FULL, 911, 4, 0.1)).astype(np.float32)
    ka_full = (1.0 + S.normal_f32(TP_K_FULL, 911, 5, 0.1)).astype(np.float32)
    qa = np.ascontiguousarray(qa_full[rank * TP_Q_LOCAL:(rank + 1) * TP_Q_LOCAL])
    ka = np.ascontiguousarray(ka_full[rank * TP_KV_LOCAL:(rank + 1) * TP_KV_LOCAL])
    cos, sin = S.rope_tables(ROPE_MAX_POS, ROT)
    return q, k, v, qa, ka, cos, sin
