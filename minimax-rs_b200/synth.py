"""Seeded synthetic inputs (numpy mirror of csrc/synth.cu, bit-for-bit).

The generator is a pure function of (seed, stream id, element index):

    mix64(z)     SplitMix64 output function
    key          mix64(seed * G ^ (stream + 1) * C)
    rand64(i)    mix64(key + (i + 1) * G)
    normal(i)    Irwin-Hall sum of the eight 16-bit fields of rand64(2i), rand64(2i+1),
                 centred (-262140) and scaled by f32(1 / (65536 sqrt(2/3))).

Stream ids of one MoE layer `L` (see ``layer_streams``): x, router, bias, gate, up, down,
residual.  The k-quant tensors use `stream` for the raw bytes and `stream + 0x10000` for the
per-block (d, dmin) halves.
"""
from __future__ import annotations

import numpy as np

GOLDEN = np.uint64(0x9E3779B97F4A7C15)
STREAM_MUL = np.uint64(0xD1B54A32D192ED03)
INV_STD = np.array([0x379CC471], dtype=np.uint32).view(np.float32)[0]

Q4K, Q5K = 1, 4
BLOCK_BYTES = {Q4K: 144, Q5K: 176}


def _mix64(z: np.ndarray) -> np.ndarray:
    z = np.asarray(z, dtype=np.uint64)
    with np.errstate(over="ignore"):
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    return z ^ (z >> np.uint64(31))


def stream_key(seed: int, stream: int) -> np.uint64:
    with np.errstate(over="ignore"):
        a = np.uint64(seed) * GOLDEN
        b = (np.uint64(stream) + np.uint64(1)) * STREAM_MUL
    return _mix64(np.array([a ^ b], dtype=np.uint64))[0]


def rand64(key: np.uint64, idx: np.ndarray) -> np.ndarray:
    idx = np.asarray(idx, dtype=np.uint64)
    with np.errstate(over="ignore"):
        return _mix64(key + (idx + np.uint64(1)) * GOLDEN)


def normal(key: np.uint64, idx: np.ndarray) -> np.ndarray:
    idx = np.asarray(idx, dtype=np.uint64)
    a = rand64(key, np.uint64(2) * idx)
    b = rand64(key, np.uint64(2) * idx + np.uint64(1))
    s = np.zeros(idx.shape, dtype=np.int64)
    for f in range(4):
        sh = np.uint64(16 * f)
        s += ((a >> sh) & np.uint64(0xFFFF)).astype(np.int64)
        s += ((b >> sh) & np.uint64(0xFFFF)).astype(np.int64)
    return (s - 262140).astype(np.float32) * INV_STD


def round_bf16(v: np.ndarray) -> np.ndarray:
    b = np.asarray(v, dtype=np.float32).view(np.uint32).astype(np.uint64)
    b = (b + np.uint64(0x7FFF) + ((b >> np.uint64(16)) & np.uint64(1))) & np.uint64(0xFFFF0000)
    return b.astype(np.uint32).view(np.float32)


def normal_f32(n: int, seed: int, stream: int, scale: float = 1.0, bf16: bool = False) -> np.ndarray:
    """scale * N(0,1), optionally rounded to bf16 — mirrors mmrs_synth_normal_f32."""
    v = normal(stream_key(seed, stream), np.arange(n, dtype=np.uint64)) * np.float32(scale)
    return round_bf16(v) if bf16 else v.astype(np.float32)


def kquant(gguf_type: int, seed: int, stream: int, experts: int, rows: int, k: int,
           row0: int = 0, nrows: int | None = None, kblk0: int = 0, nkblk: int | None = None,
           expert_ids=None) -> np.ndarray:
    """Window of a synthetic k-quant tensor [experts][rows][k/256] — mirrors mmrs_synth_kquant.

    Returns uint8 of shape [experts, nrows, nkblk * block_bytes]; with `expert_ids`, only those
    experts' windows, stacked in the given order (shape [len(expert_ids), nrows, ...])."""
    nblk = k // 256
    nrows = rows - row0 if nrows is None else nrows
    nkblk = nblk - kblk0 if nkblk is None else nkblk
    wpb = BLOCK_BYTES[gguf_type] // 8
    key = stream_key(seed, stream)
    key_d = stream_key(seed, stream + 0x10000)
    ids = np.arange(experts, dtype=np.int64) if expert_ids is None else np.asarray(expert_ids, dtype=np.int64)
    e = ids[:, None, None]
    r = np.arange(nrows, dtype=np.int64)[None, :, None]
    b = np.arange(nkblk, dtype=np.int64)[None, None, :]
    gblk = (e * rows + row0 + r) * nblk + kblk0 + b  # [E, nrows, nkblk]
    words = rand64(key, (gblk[..., None] * wpb + np.arange(wpb)).astype(np.uint64))
    d = (np.abs(normal(key_d, (2 * gblk).astype(np.uint64))) * np.float32(0.01)).astype(np.float16)
    dm = (np.abs(normal(key_d, (2 * gblk + 1).astype(np.uint64))) * np.float32(0.01)).astype(np.float16)
    low = d.view(np.uint16).astype(np.uint64) | (dm.view(np.uint16).astype(np.uint64) << np.uint64(16))
    words[..., 0] = (words[..., 0] & np.uint64(0xFFFFFFFF00000000)) | low
    return words.view(np.uint8).reshape(len(ids), nrows, nkblk * BLOCK_BYTES[gguf_type])


def q8_0_blocks(seed: int, stream: int, rows: int, k: int) -> np.ndarray:
    """Synthetic GGUF Q8_0 matrix [rows][k/32] x 34 bytes (half d = |N(0,1)| * 0.01, then 32
    uniform int8 quants), as uint8 [rows, k/32 * 34]."""
    nb = k // 32
    key, key_d = stream_key(seed, stream), stream_key(seed, stream + 0x10000)
    blk = np.arange(rows * nb, dtype=np.uint64)
    q = rand64(key, (blk[:, None] * np.uint64(4) + np.arange(4, dtype=np.uint64)).ravel()).view(np.uint8)
    d = (np.abs(normal(key_d, blk)) * np.float32(0.01)).astype(np.float16)
    out = np.empty((rows * nb, 34), dtype=np.uint8)
    out[:, :2] = d.view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q.reshape(-1, 32)
    return out.reshape(rows, nb * 34)


def q6k_blocks(seed: int, stream: int, rows: int, k: int) -> np.ndarray:
    """Synthetic GGUF Q6_K matrix [rows][k/256] x 210 bytes: ql (128 B) and qh (64 B) uniform
    bytes, 16 int8 scales uniform in [-64, 63], half d = |N(0,1)| * 0.002, as uint8 [rows, k/256 * 210]."""
    nb = k // 256
    key, key_d = stream_key(seed, stream), stream_key(seed, stream + 0x10000)
    blk = np.arange(rows * nb, dtype=np.uint64)
    q = rand64(key, (blk[:, None] * np.uint64(26) + np.arange(26, dtype=np.uint64)).ravel()).view(np.uint8)
    q = q.reshape(-1, 208)
    d = (np.abs(normal(key_d, blk)) * np.float32(0.002)).astype(np.float16)
    out = np.empty((rows * nb, 210), dtype=np.uint8)
    out[:, :192] = q[:, :192]
    out[:, 192:208] = ((q[:, 192:208].astype(np.int16) & 127) - 64).astype(np.int8).view(np.uint8)
    out[:, 208:] = d.view(np.uint8).reshape(-1, 2)
    return out.reshape(rows, nb * 210)


def normal_f16(n: int, seed: int, stream: int, scale: float = 1.0) -> np.ndarray:
    """scale * N(0,1) rounded to half (round to nearest even)."""
    return normal_f32(n, seed, stream, scale).astype(np.float16)


def rope_tables(max_pos: int, rope_dim: int, theta: float = 5.0e6):
    """cos / sin [max_pos][rope_dim / 2] f32 of the rotary embedding: angle(p, i) = p * theta^(-2i/rope_dim)."""
    inv = theta ** (-np.arange(0, rope_dim, 2, dtype=np.float64) / rope_dim)
    ang = np.arange(max_pos, dtype=np.float64)[:, None] * inv[None, :]
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def layer_streams(layer: int) -> dict:
    base = 16 * layer
    return dict(x=base + 0, router=base + 1, bias=base + 2, gate=base + 3, up=base + 4,
                down=base + 5, residual=base + 6)


def zipf_bias(num_experts: int, seed: int, s: float = 1.1, kappa: float = 0.065) -> np.ndarray:
    """Correction bias that skews top-k hits towards a Zipf(s) popularity over a seeded
    permutation of the experts: bias_e = -kappa * s * ln(1 + rank_e).  kappa = 0.065 is
    calibrated for T = 512 tokens x ~ N(0, 1) and a router ~ N(0, 0.02): per-expert
    route counts span 0 to ~190 and ~225 of the 256 experts are touched."""
    key = stream_key(seed, 0x7A1F)
    perm = np.argsort(rand64(key, np.arange(num_experts, dtype=np.uint64)), kind="stable")
    rank = np.empty(num_experts, dtype=np.int64)
    rank[perm] = np.arange(num_experts)
    return (-kappa * s * np.log1p(rank.astype(np.float64))).astype(np.float32)
