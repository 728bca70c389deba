"""LM head on the GPU against the reference kernel's recorded logits (tests/golden/ref_lmhead.npz)
and the CPU oracle: the reference-named Q6_K launcher, and the fused output_norm + Q6_K matvec +
greedy token (odd row counts, ties, a large vocabulary slice)."""
from __future__ import annotations

import ctypes as C
import sys
from pathlib import Path

import numpy as np
import pytest

sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
import golden_cases as G  # noqa: E402

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).resolve().parent / "golden" / "ref_lmhead.npz"


def _rel(a, b) -> float:
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def _s():
    import torch
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def test_q6k_plain_launcher_matches_reference(pkg, orc, dev):
    """launch_mmvq_gguf_quantize_q8_1_f32 + launch_mmvq_gguf_q6_k_f32_plain (b_size 1)."""
    import torch
    L = pkg.lib()
    gold = np.load(GOLD)
    x, w = G.lm_inputs()
    xd, wd = torch.from_numpy(x).to(dev), torch.from_numpy(np.ascontiguousarray(w)).to(dev)
    vy = torch.zeros(G.LM_K // 32 * 36, dtype=torch.uint8, device=dev)
    y = torch.zeros(G.LM_ROWS, dtype=torch.float32, device=dev)
    L.launch_mmvq_gguf_quantize_q8_1_f32(C.c_void_p(xd.data_ptr()), C.c_void_p(vy.data_ptr()), G.LM_K, G.LM_K, 1,
                                         _s())
    L.launch_mmvq_gguf_q6_k_f32_plain(C.c_void_p(wd.data_ptr()), C.c_void_p(vy.data_ptr()),
                                      C.c_void_p(y.data_ptr()), G.LM_K, G.LM_ROWS, G.LM_K // 32, G.LM_ROWS, 1, _s())
    torch.cuda.synchronize()
    assert pkg.last_error() == 0
    got = y.cpu().numpy()
    assert _rel(got, gold["logits"]) < 1e-6
    assert _rel(got, orc.q6k_matvec(w, G.LM_ROWS, G.LM_K, x)) < 1e-6
    # the Q8_1 scratch holds the reference's block layout
    ref_q = gold["vy"].reshape(-1, 36)
    got_q = vy.cpu().numpy().reshape(-1, 36)
    assert np.array_equal(got_q[:, :2], ref_q[:, :2]) and np.array_equal(got_q[:, 4:], ref_q[:, 4:])


def _norm_ref(x, w, eps=1e-6):
    x64 = x.astype(np.float64)
    return (x64 / np.sqrt(np.mean(x64 * x64) + eps) * w).astype(np.float32)


@pytest.mark.parametrize("rows", [4096, 1001, 50016])
def test_fused_head_matches_oracle(pkg, orc, synth, dev, rows):
    """output_norm + Q8_1 + Q6_K matvec + greedy token: logits within 1e-5 of the oracle chain, the
    token equal to the oracle's argmax; 1001 rows exercises the odd last row; repeated calls leave
    the workspace's counters at zero (identical second result)."""
    import torch
    k = 3072
    w = synth.q6k_blocks(911, 2, rows, k)
    x = synth.normal_f32(k, 911, 3, 3.0)
    nw = (1.0 + synth.normal_f32(k, 911, 4, 0.1)).astype(np.float32)
    head = pkg.LmHead(torch.from_numpy(np.ascontiguousarray(w)).to(dev), torch.from_numpy(nw).to(dev), rows, k)
    xd = torch.from_numpy(x).to(dev)
    lg1, tok1 = head.forward(xd)
    lg1, t1 = lg1.cpu().numpy().copy(), int(tok1.item())
    lg2, tok2 = head.forward(xd)
    torch.cuda.synchronize()
    assert head.status() == 0
    assert np.array_equal(lg1, lg2.cpu().numpy()) and t1 == int(tok2.item())
    ref = orc.q6k_matvec(w, rows, k, _norm_ref(x, nw))
    assert _rel(lg1, ref) < 1e-5
    assert t1 == orc.argmax_f32(lg1)
    assert t1 == orc.argmax_f32(ref)


def test_greedy_token_takes_the_first_of_equal_maxima(pkg, synth, dev):
    """Rows 7 and 3000 are copies of the row with the largest logit: the token is the lowest of the
    three indices (the reference's argmax keeps the first maximum)."""
    import torch
    rows, k = 4096, 3072
    w = synth.q6k_blocks(913, 2, rows, k)
    x = synth.normal_f32(k, 913, 3, 1.0)
    head = pkg.LmHead(torch.from_numpy(np.ascontiguousarray(w)).to(dev), None, rows, k)
    lg, _ = head.forward(torch.from_numpy(x).to(dev))
    best = int(np.argmax(lg.cpu().numpy()))
    w2 = w.copy()
    w2[7] = w[best]
    w2[3000] = w[best]
    head2 = pkg.LmHead(torch.from_numpy(np.ascontiguousarray(w2)).to(dev), None, rows, k)
    lg2, tok = head2.forward(torch.from_numpy(x).to(dev))
    torch.cuda.synchronize()
    l2 = lg2.cpu().numpy()
    assert l2[7] == l2[best] == l2[3000]
    assert int(tok.item()) == min(7, best)
