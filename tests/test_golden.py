"""The CPU oracle against the reference's own kernels (golden vectors, tests/golden/README.md)."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
import golden_cases as G  # noqa: E402

GOLD = np.load(Path(__file__).resolve().parent / "golden" / "ref_kernels.npz")


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


@pytest.mark.parametrize("name,gt", [("q4k", G.Q4K), ("q5k", G.Q5K)])
def test_dequant_bit_exact(orc, name, gt):
    ref = GOLD[f"dequant_{name}"]
    out = orc.dequant(gt, G.dequant_blocks(gt), fused=True)
    assert np.array_equal(out.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("kx", G.QUANT_K)
def test_quantize_q8_1_bytes(orc, kx):
    assert np.array_equal(orc.quantize_q8_1(G.quant_input(kx)).reshape(-1), GOLD[f"q81_k{kx}"])


def test_quantize_mmq_ds4_bytes(orc):
    x, ids, kx, div = G.mmq_quant_case()
    kpad = (kx + 511) // 512 * 512
    q, d, s = orc.quantize_q8_1_mmq(x, ids // div, kpad=kpad)
    rq, rd, rs = G.mmq_layout_to_logical(GOLD["mmq_q81"], len(ids), kpad)
    assert np.array_equal(q, rq) and np.array_equal(d, rd) and np.array_equal(s, rs)


def test_decode_topk(orc):
    lg, bias = G.topk_inputs()
    for i in range(lg.shape[0]):
        ids, w, e, r = orc.decode_topk(lg[i], bias)
        assert np.array_equal(ids, GOLD["topk_ids"][i])
        assert np.array_equal(e, GOLD["topk_experts"][i])
        assert np.array_equal(r, GOLD["topk_routes"][i])
        ulp = np.abs(w.view(np.int32).astype(np.int64) - GOLD["topk_w"][i].view(np.int32).astype(np.int64))
        assert ulp.max() <= 2
    # the planted tie (experts 10 and 20, equal scores) resolves to the lower id first
    assert list(GOLD["topk_ids"][0][:2]) == [10, 20]


@pytest.mark.parametrize("c", G.DECODE_CASES, ids=lambda c: c["name"])
def test_decode_silu(orc, c):
    L = G.layer(c)
    routes, experts, w = G.decode_routing(c)
    y = orc.moe_decode_silu(G.token(c), L["gate"], L["up"], L["down"], routes, experts, w, c["E"], c["H"], c["I"],
                            c["gu"], c["dn"])
    assert rel(y, GOLD[f"decode_{c['name']}"]) < 1e-6


@pytest.mark.parametrize("c", G.GEMM_CASES, ids=lambda c: c["name"])
def test_expert_gemm(orc, c):
    inp, w, sorted_ids, experts, tw = G.gemm_inputs(c)
    out = orc.moe_gemm_gguf(inp, w, sorted_ids, experts, tw, c["E"], 8, c["M"], c["N"], c["K"], c["type"],
                            mmq=c["mmq"])
    assert rel(out, GOLD[f"gemm_{c['name']}"].reshape(c["M"], c["N"])) < 1e-6


def test_sort_routes_stable(orc):
    se, sr = orc.sort_routes(G.sort_input())
    assert np.array_equal(se, GOLD["sort_experts"]) and np.array_equal(sr, GOLD["sort_routes"])
