"""Decode attention on the GPU against the reference kernels' recorded outputs
(tests/golden/ref_attn.npz) and the CPU oracle: the reference-named launchers one by one, then the
fused single-token forward (projection, RMSNorm, RoPE, KV append, GQA, output projection)."""
from __future__ import annotations

import ctypes as C
import math
import sys
from pathlib import Path

import numpy as np
import pytest

sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
import golden_cases as G  # noqa: E402

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).resolve().parent / "golden" / "ref_attn.npz"


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLD)


def _rel(a, b) -> float:
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def _f16(bits) -> np.ndarray:
    return np.asarray(bits).view(np.float16).astype(np.float64)


def _ulps(a_bits, b_bits) -> np.ndarray:
    return np.abs(np.asarray(a_bits).view(np.int16).astype(np.int32) - np.asarray(b_bits).view(np.int16).astype(np.int32))


def _t(pkg, a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _s():
    import torch
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def test_qkv_rmsnorm_matches_reference_and_oracle(pkg, orc, dev, gold):
    import torch
    L = pkg.lib()
    x, wq, wk, wv, qa, ka = G.qkv_inputs()
    n = G.Q_ROWS + G.K_ROWS + G.V_ROWS
    t = [_t(pkg, a, dev) for a in (x, wq, wk, wv, qa, ka)]
    vy = torch.zeros(G.ATTN_H // 32 * 36, dtype=torch.uint8, device=dev)
    proj = torch.zeros(n, dtype=torch.float32, device=dev)
    out = torch.zeros(n, dtype=torch.float16, device=dev)
    P = lambda a: C.c_void_p(a.data_ptr())  # noqa: E731
    L.launch_mmvq_gguf_qkv_q8_0_f32_rmsnorm_f16(P(t[0]), P(vy), P(t[1]), P(t[2]), P(t[3]), P(proj), P(t[4]), P(t[5]),
                                                P(out), G.ATTN_H, G.ATTN_H, G.Q_ROWS, G.K_ROWS, G.V_ROWS, 1e-6, _s())
    torch.cuda.synchronize()
    assert pkg.last_error() == 0
    p = proj.cpu().numpy()
    assert _rel(p, gold["qkv_proj"]) < 1e-6
    assert np.max(np.abs(p - gold["qkv_proj"])) < 1e-5 * np.max(np.abs(gold["qkv_proj"]))
    ob = out.cpu().numpy().view(np.uint16)
    assert _ulps(ob, gold["qkv_f16"]).max() <= 1
    assert np.mean(ob == gold["qkv_f16"]) > 0.9
    assert _ulps(ob, orc.qkv_rmsnorm_f16(p, qa, ka, G.Q_ROWS, G.K_ROWS, G.V_ROWS, 1e-6)).max() <= 1
    # the Q8_1 scratch holds the reference's block layout (half d, half sum, 32 int8)
    ref_q = orc.quantize_q8_1(x.reshape(1, -1), G.ATTN_H).reshape(-1, 36)
    got_q = vy.cpu().numpy().reshape(-1, 36)
    assert np.array_equal(got_q[:, :2], ref_q[:, :2]) and np.array_equal(got_q[:, 4:], ref_q[:, 4:])


@pytest.mark.parametrize("pos", G.ROPE_POS)
def test_partial_rope_bit_exact(pkg, dev, gold, pos):
    import torch
    L = pkg.lib()
    q, k, cos, sin = G.rope_inputs()
    t = [_t(pkg, a, dev) for a in (q, k, cos, sin)]
    out = torch.zeros(G.Q_ROWS + G.K_ROWS, dtype=torch.float16, device=dev)
    L.launch_partial_rope_f16(*[C.c_void_p(a.data_ptr()) for a in t], C.c_void_p(out.data_ptr()), G.Q_ROWS, G.K_ROWS,
                              G.HD, G.ROT, pos, _s())
    torch.cuda.synchronize()
    assert pkg.last_error() == 0
    assert np.array_equal(out.cpu().numpy().view(np.uint16), gold[f"rope_p{pos}"])


@pytest.mark.parametrize("seq_len,splits", G.GQA_CASES + ((1000, 1), (4096, 128), (37, 40)))
def test_gqa_decode(pkg, orc, dev, gold, seq_len, splits):
    """Against the exact oracle to f16 rounding, and against the reference's f16 tensor-core kernel
    (f16 probabilities) to ~1e-3; empty splits (more splits than keys) included."""
    import torch
    L = pkg.lib()
    q, k, v = G.gqa_inputs(seq_len)
    t = [_t(pkg, a, dev) for a in (q, k, v)]
    part = torch.zeros(splits * G.QH * (G.HD + 2), dtype=torch.float32, device=dev)
    out = torch.zeros(G.QH * G.HD, dtype=torch.float16, device=dev)
    scale = 1.0 / math.sqrt(G.HD)
    L.launch_gqa_decode_mma_f16_128(*[C.c_void_p(a.data_ptr()) for a in t], C.c_void_p(part.data_ptr()),
                                    C.c_void_p(out.data_ptr()), seq_len, G.HD, G.KV_CAP * G.HD, G.KV_CAP * G.HD,
                                    splits, G.QH, G.KVH, scale, 0, _s())
    torch.cuda.synchronize()
    assert pkg.last_error() == 0
    got = out.cpu().numpy().view(np.uint16)
    ref = orc.gqa_decode_f16(q, k, v, seq_len, G.QH, G.KVH, G.HD, G.KV_CAP * G.HD, scale)
    assert _rel(_f16(got), _f16(ref)) < 5e-4
    assert _ulps(got, ref).max() <= 4
    key = f"gqa_s{seq_len}_n{splits}"
    if key in gold.files:
        assert _rel(_f16(got), _f16(gold[key])) < 2e-3


def test_output_projection_matches_reference(pkg, orc, dev, gold):
    """launch_mmvq_gguf_quantize_q8_1_f32 + launch_mmvq_gguf_q8_0_f32_plain (b_size 1)."""
    import torch
    L = pkg.lib()
    a, wo = G.oproj_inputs()
    ad, wd = _t(pkg, a, dev), _t(pkg, wo, dev)
    vy = torch.zeros(G.Q_ROWS // 32 * 36, dtype=torch.uint8, device=dev)
    y = torch.zeros(G.ATTN_H, dtype=torch.float32, device=dev)
    L.launch_mmvq_gguf_quantize_q8_1_f32(C.c_void_p(ad.data_ptr()), C.c_void_p(vy.data_ptr()), G.Q_ROWS, G.Q_ROWS, 1,
                                         _s())
    L.launch_mmvq_gguf_q8_0_f32_plain(C.c_void_p(wd.data_ptr()), C.c_void_p(vy.data_ptr()), C.c_void_p(y.data_ptr()),
                                      G.Q_ROWS, G.ATTN_H, G.Q_ROWS // 32, G.ATTN_H, 1, _s())
    torch.cuda.synchronize()
    assert pkg.last_error() == 0
    got = y.cpu().numpy()
    assert _rel(got, gold["oproj"]) < 1e-6
    assert _rel(got, orc.q8_0_matvec(wo, G.ATTN_H, G.Q_ROWS, a)) < 1e-6


def test_unsupported_batch_is_reported(pkg, dev):
    import torch
    L = pkg.lib()
    z = torch.zeros(64, dtype=torch.uint8, device=dev)
    L.launch_mmvq_gguf_q8_0_f32_plain(C.c_void_p(z.data_ptr()), C.c_void_p(z.data_ptr()), C.c_void_p(z.data_ptr()),
                                      64, 1, 2, 1, 2, _s())
    assert pkg.last_error() == pkg.MMRS_ERR_UNSUPPORTED


def _layer(pkg, dev, hidden, seed, max_pos=64):
    import torch
    S = G.S
    qr, kr = G.Q_ROWS, G.K_ROWS
    w = dict(wq=S.q8_0_blocks(seed, 2, qr, hidden), wk=S.q8_0_blocks(seed, 3, kr, hidden),
             wv=S.q8_0_blocks(seed, 4, kr, hidden), wo=S.q8_0_blocks(seed, 5, hidden, qr),
             qn=(1.0 + S.normal_f32(qr, seed, 6, 0.1)).astype(np.float32),
             kn=(1.0 + S.normal_f32(kr, seed, 7, 0.1)).astype(np.float32))
    cos, sin = S.rope_tables(max_pos, G.ROT)
    t = {k: torch.from_numpy(v).to(dev) for k, v in w.items()}
    layer = pkg.AttnLayer(t["wq"], t["wk"], t["wv"], t["wo"], t["qn"], t["kn"], torch.from_numpy(cos).to(dev),
                          torch.from_numpy(sin).to(dev), hidden)
    return layer, w, cos, sin


def test_fused_decode_steps_match_oracle(pkg, orc, dev):
    """Five decode steps through mmrs_attn_decode_forward (K / V appended to the cache at each
    position) against the oracle's chain of the same operations."""
    import torch
    hidden, seed, steps = G.ATTN_H, 801, 5
    layer, w, cos, sin = _layer(pkg, dev, hidden, seed)
    xs = G.S.normal_f32(steps * hidden, seed, 8, 1.0).reshape(steps, hidden)
    res = G.S.normal_f32(hidden, seed, 9, 1.0)
    qr, kr = G.Q_ROWS, G.K_ROWS
    kc = np.zeros((G.KVH, 64, G.HD), dtype=np.uint16)
    vc = np.zeros_like(kc)
    for pos in range(steps):
        y = layer.forward(torch.from_numpy(xs[pos]).to(dev), pos, residual=torch.from_numpy(res).to(dev))
        torch.cuda.synchronize()
        # oracle chain
        proj = np.concatenate([orc.q8_0_matvec(w["wq"], qr, hidden, xs[pos]), orc.q8_0_matvec(w["wk"], kr, hidden, xs[pos]),
                               orc.q8_0_matvec(w["wv"], kr, hidden, xs[pos])])
        nrm = orc.qkv_rmsnorm_f16(proj, w["qn"], w["kn"], qr, kr, kr, 1e-6)
        rot = orc.partial_rope_f16(nrm[:qr], nrm[qr:qr + kr], cos, sin, G.HD, G.ROT, pos)
        kc[:, pos] = rot[qr:].reshape(G.KVH, G.HD)
        vc[:, pos] = nrm[qr + kr:].reshape(G.KVH, G.HD)
        att = orc.gqa_decode_f16(rot[:qr], kc, vc, pos + 1, G.QH, G.KVH, G.HD, 64 * G.HD, 1.0 / math.sqrt(G.HD))
        ref = orc.q8_0_matvec(w["wo"], hidden, qr, _f16(att).astype(np.float32)) + res
        got = y.cpu().numpy()
        assert _rel(got - res, ref - res) < 5e-3, pos
        # the caches hold the rotated K and the V of every step so far
        assert _ulps(layer.k_cache[:, pos].cpu().numpy().view(np.uint16), kc[:, pos]).max() <= 2
        assert _ulps(layer.v_cache[:, pos].cpu().numpy().view(np.uint16), vc[:, pos]).max() <= 1


def _oracle_step(orc, w, x, res, kc, vc, cos, sin, pos, hidden):
    qr, kr = G.Q_ROWS, G.K_ROWS
    proj = np.concatenate([orc.q8_0_matvec(w["wq"], qr, hidden, x), orc.q8_0_matvec(w["wk"], kr, hidden, x),
                           orc.q8_0_matvec(w["wv"], kr, hidden, x)])
    nrm = orc.qkv_rmsnorm_f16(proj, w["qn"], w["kn"], qr, kr, kr, 1e-6)
    rot = orc.partial_rope_f16(nrm[:qr], nrm[qr:qr + kr], cos, sin, G.HD, G.ROT, pos)
    kc[:, pos] = rot[qr:].reshape(G.KVH, G.HD)
    vc[:, pos] = nrm[qr + kr:].reshape(G.KVH, G.HD)
    att = orc.gqa_decode_f16(rot[:qr], kc, vc, pos + 1, G.QH, G.KVH, G.HD, kc.shape[1] * G.HD, 1.0 / math.sqrt(G.HD))
    return orc.q8_0_matvec(w["wo"], hidden, qr, _f16(att).astype(np.float32)) + res


@pytest.mark.parametrize("pos", [700, 1023])
def test_fused_decode_long_cache(pkg, orc, dev, pos):
    """A step at a late position over a filled cache: several key splits merged by the last CTA of
    each KV head, the new position inside a chunk (700) or closing the cache (1023).  The step runs
    twice: the split counters return to zero, so the second result is identical."""
    import torch
    hidden, seed, cap = G.ATTN_H, 811, 1024
    layer, w, cos, sin = _layer(pkg, dev, hidden, seed, max_pos=cap)
    kc = G.S.normal_f16(G.KVH * cap * G.HD, seed, 10, 1.0).reshape(G.KVH, cap, G.HD).view(np.uint16).copy()
    vc = G.S.normal_f16(G.KVH * cap * G.HD, seed, 11, 1.0).reshape(G.KVH, cap, G.HD).view(np.uint16).copy()
    layer.k_cache.copy_(torch.from_numpy(kc.view(np.float16)))
    layer.v_cache.copy_(torch.from_numpy(vc.view(np.float16)))
    x = G.S.normal_f32(hidden, seed, 8, 1.0)
    res = G.S.normal_f32(hidden, seed, 9, 1.0)
    xd, rd = torch.from_numpy(x).to(dev), torch.from_numpy(res).to(dev)
    y1 = layer.forward(xd, pos, residual=rd).cpu().numpy()
    y2 = layer.forward(xd, pos, residual=rd).cpu().numpy()
    torch.cuda.synchronize()
    assert layer.status() == 0
    assert np.array_equal(y1, y2)
    ref = _oracle_step(orc, w, x, res, kc, vc, cos, sin, pos, hidden)
    assert _rel(y1 - res, ref - res) < 5e-3
    assert _ulps(layer.k_cache[:, pos].cpu().numpy().view(np.uint16), kc[:, pos]).max() <= 2
    assert _ulps(layer.v_cache[:, pos].cpu().numpy().view(np.uint16), vc[:, pos]).max() <= 1
    # positions other than `pos` are untouched
    got_k = layer.k_cache.cpu().numpy().view(np.uint16)
    keep = np.ones(cap, bool)
    keep[pos] = False
    assert np.array_equal(got_k[:, keep], kc[:, keep])


def test_rmsnorm_rows(pkg, synth, dev):
    import torch
    x = synth.normal_f32(3 * 3072, 901, 1, 2.0).reshape(3, 3072)
    w = (1.0 + synth.normal_f32(3072, 901, 2, 0.1)).astype(np.float32)
    y = pkg.rmsnorm(torch.from_numpy(x).to(dev), torch.from_numpy(w).to(dev), eps=1e-6)
    torch.cuda.synchronize()
    x64 = x.astype(np.float64)
    ref = x64 / np.sqrt(np.mean(x64 * x64, axis=1, keepdims=True) + 1e-6) * w
    assert _rel(y.cpu().numpy(), ref) < 1e-6


def test_streaming_matvec_refills_the_ring(pkg, orc, synth, dev):
    """A Q8_0 matrix of 24576 x 3072 (about 33 groups of rows per CTA, so every slot of the
    12-slot ring is refilled): against the oracle, and bit-identical across repeated calls."""
    import torch
    L = pkg.lib()
    rows, k = 24576, 3072
    w = synth.q8_0_blocks(931, 2, rows, k)
    x = synth.normal_f32(k, 931, 3, 1.0)
    wd, xd = torch.from_numpy(np.ascontiguousarray(w)).to(dev), torch.from_numpy(x).to(dev)
    vy = torch.zeros(k // 32 * 36, dtype=torch.uint8, device=dev)
    L.launch_mmvq_gguf_quantize_q8_1_f32(C.c_void_p(xd.data_ptr()), C.c_void_p(vy.data_ptr()), k, k, 1, _s())
    outs = []
    for _ in range(3):
        y = torch.zeros(rows, dtype=torch.float32, device=dev)
        L.launch_mmvq_gguf_q8_0_f32_plain(C.c_void_p(wd.data_ptr()), C.c_void_p(vy.data_ptr()),
                                          C.c_void_p(y.data_ptr()), k, rows, k // 32, rows, 1, _s())
        torch.cuda.synchronize()
        assert pkg.last_error() == 0
        outs.append(y.cpu().numpy())
    assert np.array_equal(outs[0], outs[1]) and np.array_equal(outs[0], outs[2])
    assert _rel(outs[0], orc.q8_0_matvec(w, rows, k, x)) < 1e-6
