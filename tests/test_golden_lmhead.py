"""The CPU oracle of the LM head against the reference kernel's own outputs
(tests/golden/ref_lmhead.npz, recorded by tests/golden/make_golden_lmhead.py on a B200 from the
reference's mmvq_gguf.cu: quantize_q8_1 + the Q6_K matvec)."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
import golden_cases as G  # noqa: E402

GOLD = Path(__file__).resolve().parent / "golden" / "ref_lmhead.npz"


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLD)


def _rel(a, b) -> float:
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def test_q6k_matvec_matches_reference(orc, gold):
    """Q6_K x Q8_1: the oracle is exact up to its final rounding; the reference sums per-thread
    float partials (MMVQ), so the two agree to float rounding; both pick the same token."""
    x, w = G.lm_inputs()
    y = orc.q6k_matvec(w, G.LM_ROWS, G.LM_K, x)
    ref = gold["logits"]
    assert _rel(y, ref) < 1e-6
    assert np.max(np.abs(y - ref)) < 1e-5 * np.max(np.abs(ref))
    assert orc.argmax_f32(y) == int(np.argmax(ref))


def test_activation_q8_1_bytes_match_reference(orc, gold):
    """The reference's quantize_q8_1 output: d and the quants bit for bit (the half sum is a
    tree sum in the reference's lane order)."""
    x, _ = G.lm_inputs()
    ref = gold["vy"].reshape(-1, 36)
    got = orc.quantize_q8_1(x.reshape(1, -1), G.LM_K).reshape(-1, 36)
    assert np.array_equal(got[:, :2], ref[:, :2]) and np.array_equal(got[:, 4:], ref[:, 4:])


def test_q6k_dequant_is_the_block_layout(orc, synth):
    """Dequantisation of one super-block against the layout written out element by element
    (ql low / high nibbles, qh 2-bit fields, 16-element int8 scales, half d)."""
    blk = synth.q6k_blocks(3, 4, 1, 256)[0]
    ql, qh, sc = blk[:128], blk[128:192], blk[192:208].view(np.int8)
    d = float(blk[208:210].view(np.float16)[0])
    want = np.zeros(256)
    for half in range(2):
        for l in range(32):
            for q in range(4):
                low = ql[64 * half + l + (q & 1) * 32]
                v = ((low & 0xF) if q < 2 else (low >> 4)) | (((qh[32 * half + l] >> (2 * q)) & 3) << 4)
                e = 128 * half + 32 * q + l
                want[e] = d * float(sc[e // 16]) * (int(v) - 32)
    got = orc.q6k_dequant_row(blk, 256)
    assert np.allclose(got, want, rtol=0, atol=1e-6 * np.abs(want).max())


def test_argmax_first_maximum(orc):
    v = np.array([1.0, 5.0, -2.0, 5.0, np.nan, 4.0], np.float32)
    assert orc.argmax_f32(v) == 1
    assert orc.argmax_f32(np.array([np.nan, -1.0], np.float32)) == 1
