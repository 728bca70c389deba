"""The CPU oracle of the decode-attention half against the reference kernels' own outputs
(tests/golden/ref_attn.npz, recorded by tests/golden/make_golden_attn.py on a B200 from the
reference's mmvq_gguf.cu / decode_attention.cu)."""
from __future__ import annotations

import math
import sys
from pathlib import Path

import numpy as np
import pytest

sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
import golden_cases as G  # noqa: E402

GOLD = Path(__file__).resolve().parent / "golden" / "ref_attn.npz"


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLD)


def _f16(bits: np.ndarray) -> np.ndarray:
    return np.asarray(bits, dtype=np.uint16).view(np.float16).astype(np.float64)


def _rel(a, b) -> float:
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def test_q8_0_qkv_projection(orc, gold):
    """Q8_0 x Q8_1 matvec: the oracle is exact up to its final rounding; the reference sums
    per-thread float partials (MMVQ), so the two agree to float rounding."""
    x, wq, wk, wv, _, _ = G.qkv_inputs()
    y = np.concatenate([orc.q8_0_matvec(wq, G.Q_ROWS, G.ATTN_H, x), orc.q8_0_matvec(wk, G.K_ROWS, G.ATTN_H, x),
                        orc.q8_0_matvec(wv, G.V_ROWS, G.ATTN_H, x)])
    ref = gold["qkv_proj"]
    assert _rel(y, ref) < 1e-6
    assert np.max(np.abs(y - ref)) < 1e-5 * np.max(np.abs(ref))


def test_qkv_rmsnorm_f16(orc, gold):
    """Given the reference's projection, RMSNorm + f16 agree to one f16 ulp (rsqrtf vs exact)."""
    _, _, _, _, qa, ka = G.qkv_inputs()
    out = orc.qkv_rmsnorm_f16(gold["qkv_proj"], qa, ka, G.Q_ROWS, G.K_ROWS, G.V_ROWS, 1e-6)
    ref = gold["qkv_f16"]
    ulp = np.abs(out.view(np.int16).astype(np.int32) - ref.view(np.int16).astype(np.int32))
    assert ulp.max() <= 1
    assert np.array_equal(out[G.Q_ROWS + G.K_ROWS:], ref[G.Q_ROWS + G.K_ROWS:])  # V: plain f16 rounding
    assert np.mean(ulp == 0) > 0.9


@pytest.mark.parametrize("pos", G.ROPE_POS)
def test_partial_rope_bit_exact(orc, gold, pos):
    q, k, cos, sin = G.rope_inputs()
    out = orc.partial_rope_f16(q, k, cos, sin, G.HD, G.ROT, pos)
    assert np.array_equal(out, gold[f"rope_p{pos}"])


@pytest.mark.parametrize("seq_len,splits", G.GQA_CASES)
def test_gqa_decode(orc, gold, seq_len, splits):
    """Exact softmax attention (double) against the reference's f16 tensor-core kernel, whose
    probabilities are rounded to f16 before the P.V product: agreement to ~1e-3."""
    q, k, v = G.gqa_inputs(seq_len)
    out = orc.gqa_decode_f16(q, k, v, seq_len, G.QH, G.KVH, G.HD, G.KV_CAP * G.HD, 1.0 / math.sqrt(G.HD))
    ref = _f16(gold[f"gqa_s{seq_len}_n{splits}"])
    assert _rel(_f16(out), ref) < 2e-3
    if seq_len == 1:  # one key: the output is that key's V row (up to f16 rounding)
        assert np.max(np.abs(_f16(out) - ref)) <= 2e-3


def test_q8_0_output_projection(orc, gold):
    a, wo = G.oproj_inputs()
    y = orc.q8_0_matvec(wo, G.ATTN_H, G.Q_ROWS, a)
    assert _rel(y, gold["oproj"]) < 1e-6
