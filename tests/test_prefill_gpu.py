"""Multi-token path through the C ABI: route sort, the generic and MMQ expert GEMMs and the
fused block for T > 1, against the reference's golden outputs and the CPU oracle."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

from moe_cases import make_layer

sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
import golden_cases as G  # noqa: E402

pytestmark = pytest.mark.gpu
GOLD = np.load(Path(__file__).resolve().parent / "golden" / "ref_kernels.npz")
Q4K, Q5K = 1, 4


def _d(dev, a):
    import torch
    return None if a is None else torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def test_sort_routes_vs_reference(pkg, dev):
    keys = G.sort_input()
    se, sr = pkg.sort_routes(_d(dev, keys.view(np.int32)), 8)
    assert np.array_equal(se.cpu().numpy().view(np.uint32), GOLD["sort_experts"])
    assert np.array_equal(sr.cpu().numpy().view(np.uint32), GOLD["sort_routes"])


@pytest.mark.parametrize("n,end_bit,high", [(1, 1, False), (7, 3, False), (1000, 8, False), (5003, 10, False),
                                            (4096, 9, False), (3000, 4, True)])
def test_sort_routes_stable_edges(pkg, dev, n, end_bit, high):
    rng = np.random.default_rng(n * 31 + end_bit)
    hi = 1 << (end_bit + 3 if high else end_bit)
    keys = rng.integers(0, hi, size=n, dtype=np.int64).astype(np.uint32)
    se, sr = pkg.sort_routes(_d(dev, keys.view(np.int32)), end_bit)
    order = np.argsort(keys & np.uint32((1 << end_bit) - 1), kind="stable")
    assert np.array_equal(sr.cpu().numpy().view(np.uint32), order.astype(np.uint32))
    assert np.array_equal(se.cpu().numpy().view(np.uint32), keys[order])


def test_sort_routes_empty(pkg, dev):
    import torch
    se, sr = pkg.sort_routes(torch.empty(0, dtype=torch.int32, device=dev), 8)
    assert se.numel() == 0 and sr.numel() == 0


@pytest.mark.parametrize("c", G.GEMM_CASES, ids=lambda c: c["name"])
def test_expert_gemm_vs_reference_and_oracle(pkg, dev, orc, c):
    import torch
    inp, w, sorted_ids, experts, tw = G.gemm_inputs(c)
    out = torch.zeros(c["M"], c["N"], dtype=torch.float32, device=dev)
    pkg.moe_gemm(_d(dev, inp), _d(dev, w), _d(dev, sorted_ids), _d(dev, experts), _d(dev, tw), out, c["E"], 8,
                 c["N"], c["K"], c["type"], mmq=c["mmq"])
    got = out.cpu().numpy()
    ref = GOLD[f"gemm_{c['name']}"].reshape(c["M"], c["N"])
    assert np.linalg.norm(got - ref) / np.linalg.norm(ref) < 1e-5
    orc_out = orc.moe_gemm_gguf(inp, w, sorted_ids, experts, tw, c["E"], 8, c["M"], c["N"], c["K"], c["type"],
                                mmq=c["mmq"])
    # integer block dots are exact; only the f32 summation order differs from the oracle
    assert np.linalg.norm(got - orc_out) / np.linalg.norm(orc_out) < 1e-6


@pytest.mark.parametrize("mmq", [True, False])
@pytest.mark.parametrize("E,N,K,T,gt,down", [(32, 1536, 3072, 80, Q4K, False), (16, 200, 512, 24, Q5K, True),
                                             (256, 256, 768, 33, Q5K, True)])
def test_expert_gemm_shapes(pkg, synth, dev, orc, mmq, E, N, K, T, gt, down):
    """Full-size K, ragged N (not a multiple of the 128-row tile), many experts, tiles of 64 routes."""
    import torch
    rng = np.random.default_rng(E * 7 + N + T)
    rows_ids = []
    for t in range(T):
        r = rng.choice(E, 8, replace=False)
        if t < 70 and 3 not in r:
            r[0] = 3  # expert 3 gets more than 64 routes when T > 64 -> several route tiles
        rows_ids.append(r)
    ids = np.stack(rows_ids).astype(np.uint32)
    flat = ids.reshape(-1)
    order = np.argsort(flat, kind="stable").astype(np.int32)
    experts = flat[order].astype(np.int32)
    M = T * 8
    rows = M if down else T
    inp = synth.normal_f32(rows * K, 900 + T, 1, 3.0 if down else 1.0).reshape(rows, K)
    w = synth.kquant(gt, 901 + T, 2, E, N, K)
    tw = (np.abs(synth.normal_f32(M, 902, 3, 1.0)) * np.float32(0.2)).astype(np.float32) if down else None
    out = torch.zeros(M, N, dtype=torch.float32, device=dev)
    pkg.moe_gemm(_d(dev, inp), _d(dev, w), _d(dev, order), _d(dev, experts), _d(dev, tw), out, E, 8, N, K, gt,
                 mmq=mmq)
    got = out.cpu().numpy()
    ref = orc.moe_gemm_gguf(inp, w, order, experts, tw, E, 8, M, N, K, gt, mmq=mmq)
    assert np.linalg.norm(got - ref) / np.linalg.norm(ref) < 1e-6


def test_mmq_gemm_other_type_does_nothing(pkg, dev):
    import torch
    out = torch.full((16, 256), 7.0, device=dev)
    ids = torch.arange(16, dtype=torch.int32, device=dev)
    ex = torch.zeros(16, dtype=torch.int32, device=dev)
    inp = torch.zeros(2, 256, device=dev)
    w = torch.zeros(256 * 34, dtype=torch.uint8, device=dev)
    with pytest.raises(pkg.MoeError):
        pkg.moe_gemm(inp, w, ids, ex, None, out, 1, 8, 256, 256, 0, mmq=True)  # Q8_0: unsupported
    assert torch.all(out == 7.0)


@pytest.mark.parametrize("E,H,I,T,gu,dn,zipf", [(16, 512, 256, 4, Q4K, Q5K, False), (32, 1024, 512, 40, Q4K, Q5K, False),
                                                (16, 512, 768, 31, Q5K, Q4K, False),
                                                (256, 3072, 1536, 64, Q4K, Q5K, True)])
def test_block_forward_multi_token(pkg, synth, dev, orc, E, H, I, T, gu, dn, zipf):
    """Activations scaled to 0.05 so that every Q8_1 block sum of the down input stays inside the
    half range (with x ~ N(0, 1) and these synthetic weights they overflow: see the test below)."""
    import torch
    L = make_layer(pkg, synth, dev, E, H, I, gu, dn, seed=1100 + T, T=T, zipf=zipf, x_scale=0.05)
    layer = pkg.MoeLayer(L["router"], L["bias"], L["gate"], L["up"], L["down"], gu, dn)
    ids = torch.empty(T, 8, dtype=torch.int32, device=dev)
    wts = torch.empty(T, 8, dtype=torch.float32, device=dev)
    y = layer.forward(L["x"], residual=L["residual"], topk_ids=ids, topk_w=wts)
    torch.cuda.synchronize()
    assert layer.status() == 0
    ry, rids, rw = orc.moe_block(L["router"].cpu().numpy(), L["bias"].cpu().numpy(), L["gate"].cpu().numpy(),
                                 L["up"].cpu().numpy(), L["down"].cpu().numpy(), gu, dn, L["x"].cpu().numpy(),
                                 residual=L["residual"].cpu().numpy())
    assert np.array_equal(ids.cpu().numpy().view(np.uint32), rids)
    assert np.max(np.abs(wts.cpu().numpy() - rw) / rw) < 1e-6
    got = y.cpu().numpy()
    moe = got - L["residual"].cpu().numpy()
    rmoe = ry - L["residual"].cpu().numpy()
    assert np.linalg.norm(moe - rmoe) / np.linalg.norm(rmoe) < 1e-3


def test_block_forward_prefill_512_zipf(pkg, synth, dev, orc):
    """Config 2 (T = 512, Zipf-skewed experts) at full size: routing for all tokens against the
    oracle, outputs of a 32-token sample against the oracle block run on that sample alone (every
    token's MMQ result depends only on its own row)."""
    import torch
    E, H, I, T = 256, 3072, 1536, 512
    L = make_layer(pkg, synth, dev, E, H, I, Q4K, Q5K, seed=2002, T=T, zipf=True, x_scale=0.05)
    layer = pkg.MoeLayer(L["router"], L["bias"], L["gate"], L["up"], L["down"], Q4K, Q5K)
    ids = torch.empty(T, 8, dtype=torch.int32, device=dev)
    wts = torch.empty(T, 8, dtype=torch.float32, device=dev)
    y = layer.forward(L["x"], residual=None, topk_ids=ids, topk_w=wts)
    torch.cuda.synchronize()
    assert layer.status() == 0
    x = L["x"].cpu().numpy()
    logits = orc.router_logits(x, L["router"].cpu().numpy())
    rids, rw = orc.route_topk(logits, L["bias"].cpu().numpy())
    assert np.array_equal(ids.cpu().numpy().view(np.uint32), rids)
    counts = np.bincount(rids.reshape(-1), minlength=E)
    assert counts.max() > 64  # some expert needs several route tiles
    sample = np.arange(0, T, 16)
    ry, _, _ = orc.moe_block(L["router"].cpu().numpy(), L["bias"].cpu().numpy(), L["gate"].cpu().numpy(),
                             L["up"].cpu().numpy(), L["down"].cpu().numpy(), Q4K, Q5K, x[sample])
    got = y.cpu().numpy()[sample]
    assert np.linalg.norm(got - ry) / np.linalg.norm(ry) < 1e-3


def test_block_forward_half_overflow_matches(pkg, synth, dev, orc):
    """x ~ N(0, 1) with the synthetic weights drives the down input to ~1e4, so MMQ's half block
    sums (quantize_mmq_q8_1<DS4>) overflow to inf: the CUDA path must produce the oracle's
    non-finite pattern exactly and agree on every finite value."""
    import torch
    E, H, I, T = 32, 1024, 512, 40
    L = make_layer(pkg, synth, dev, E, H, I, Q4K, Q5K, seed=1140, T=T)
    layer = pkg.MoeLayer(L["router"], L["bias"], L["gate"], L["up"], L["down"], Q4K, Q5K)
    y = layer.forward(L["x"]).cpu().numpy()
    ry, _, _ = orc.moe_block(L["router"].cpu().numpy(), L["bias"].cpu().numpy(), L["gate"].cpu().numpy(),
                             L["up"].cpu().numpy(), L["down"].cpu().numpy(), Q4K, Q5K, L["x"].cpu().numpy())
    assert not np.all(np.isfinite(ry))
    assert np.array_equal(np.isnan(y), np.isnan(ry))
    assert np.array_equal(np.isposinf(y), np.isposinf(ry)) and np.array_equal(np.isneginf(y), np.isneginf(ry))
    f = np.isfinite(ry)
    assert np.linalg.norm(y[f] - ry[f]) / np.linalg.norm(ry[f]) < 1e-3
