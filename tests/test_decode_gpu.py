"""Single-token (decode) MoE block on the GPU against the CPU oracle."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from conftest import rel_l2
from moe_cases import make_layer, oracle_decode, expert_slices

pytestmark = pytest.mark.gpu

TOL = 1e-3  # relative L2 of the MoE block output (f32 accumulation), per the parity target


def test_synth_device_matches_numpy(pkg, synth, dev):
    import torch
    t = torch.empty(1000, dtype=torch.float32, device=dev)
    pkg.synth_normal(t, 5, 3, 0.02, bf16=False)
    assert np.array_equal(t.cpu().numpy(), synth.normal_f32(1000, 5, 3, 0.02))
    pkg.synth_normal(t, 5, 4, 1.0, bf16=True)
    assert np.array_equal(t.cpu().numpy(), synth.normal_f32(1000, 5, 4, 1.0, bf16=True))
    for gt in (pkg.Q4K, pkg.Q5K):
        bb = 144 if gt == pkg.Q4K else 176
        w = torch.empty(3 * 5 * 2 * bb, dtype=torch.uint8, device=dev)
        pkg.synth_kquant(w, gt, 9, 7, 3, 8, 1024, row0=2, nrows=5, kblk0=1, nkblk=2)
        ref = synth.kquant(gt, 9, 7, 3, 8, 1024, row0=2, nrows=5, kblk0=1, nkblk=2)
        assert np.array_equal(w.cpu().numpy(), ref.reshape(-1))


def test_decode_topk_abi_matches_oracle(pkg, orc, synth, dev):
    import torch
    lib = pkg.lib()
    for seed in range(20):
        logits = torch.from_numpy(synth.normal_f32(256, seed, 1, 1.1)).to(dev)
        bias = torch.from_numpy(synth.normal_f32(256, seed, 2, 0.01)).to(dev)
        out_ids = torch.empty(8, dtype=torch.int32, device=dev)
        out_w = torch.empty(8, dtype=torch.float32, device=dev)
        out_e = torch.empty(8, dtype=torch.int32, device=dev)
        out_r = torch.empty(8, dtype=torch.int32, device=dev)
        lib.minimax_moe_decode_topk(logits.data_ptr(), bias.data_ptr(), out_ids.data_ptr(), out_w.data_ptr(),
                                    out_e.data_ptr(), out_r.data_ptr(), torch.cuda.current_stream().cuda_stream)
        assert lib.mmrs_last_error() == 0
        ids, w, e, r = orc.decode_topk(logits.cpu().numpy(), bias.cpu().numpy())
        assert np.array_equal(out_ids.cpu().numpy().astype(np.uint32), ids)
        assert np.array_equal(out_e.cpu().numpy().astype(np.uint32), e)
        assert np.array_equal(out_r.cpu().numpy().astype(np.uint32), r)
        # CUDA expf and the host libm may differ by an ulp in the sigmoid
        np.testing.assert_allclose(out_w.cpu().numpy(), w, rtol=1e-6, atol=0)


@pytest.mark.parametrize("E,H,I,gu,dn", [(16, 512, 256, 1, 4), (256, 3072, 1536, 1, 4), (256, 3072, 768, 1, 4),
                                          (64, 3072, 1536, 1, 1)])
def test_decode_silu_abi_matches_oracle(pkg, orc, synth, dev, E, H, I, gu, dn):
    import torch
    L = make_layer(pkg, synth, dev, E, H, I, gu, dn, seed=21)
    rng = np.random.default_rng(3)
    experts = np.sort(rng.choice(E, 8, replace=False)).astype(np.int32)
    routes = rng.permutation(8).astype(np.int32)
    w = rng.random(8).astype(np.float32)
    w /= w.sum()
    y = torch.empty(H, dtype=torch.float32, device=dev)
    ex_d, rt_d, w_d = (torch.from_numpy(a).to(dev) for a in (experts, routes, w))
    pkg.lib().moe_gemm_gguf_decode_silu(L["x"].data_ptr(), L["gate"].data_ptr(), L["up"].data_ptr(),
                                        L["down"].data_ptr(), rt_d.data_ptr(), ex_d.data_ptr(), w_d.data_ptr(),
                                        y.data_ptr(), E, 8, H, I, gu, dn, torch.cuda.current_stream().cuda_stream)
    assert pkg.last_error() == 0
    g, u, d = expert_slices(pkg, L, experts)
    ref = orc.moe_decode_silu(L["x"].cpu().numpy()[0], g, u, d, routes, np.arange(8, dtype=np.int32), w, 8, H, I,
                              gu, dn)
    assert rel_l2(y.cpu().numpy(), ref) < TOL


@pytest.mark.parametrize("E,H,I,gu,dn", [(32, 1024, 512, 1, 4), (256, 3072, 1536, 1, 4), (256, 3072, 768, 1, 4),
                                          (256, 3072, 1536, 1, 1)])
def test_fused_block_decode_matches_oracle(pkg, orc, synth, dev, E, H, I, gu, dn):
    import torch
    L = make_layer(pkg, synth, dev, E, H, I, gu, dn, seed=31)
    layer = pkg.MoeLayer(L["router"], L["bias"], L["gate"], L["up"], L["down"], gu, dn)
    ids = torch.empty(1, 8, dtype=torch.int32, device=dev)
    tw = torch.empty(1, 8, dtype=torch.float32, device=dev)
    y = layer.forward(L["x"], residual=L["residual"], topk_ids=ids, topk_w=tw)
    torch.cuda.synchronize()
    assert layer.status() == 0
    ref_y, ref_ids, ref_w, _ = oracle_decode(orc, pkg, L, L["x"].cpu().numpy()[0], L["residual"].cpu().numpy()[0])
    assert np.array_equal(ids.cpu().numpy()[0].astype(np.uint32), ref_ids)
    np.testing.assert_allclose(tw.cpu().numpy()[0], ref_w, rtol=1e-6)
    assert rel_l2(y.cpu().numpy()[0], ref_y) < TOL


def test_fused_block_decode_repeatable_and_many_tokens(pkg, orc, synth, dev):
    """Consecutive launches reuse the grid-barrier state; outputs are bitwise reproducible and
    every token of a sequence of independent inputs matches the oracle."""
    import torch
    E, H, I = 256, 3072, 1536
    L = make_layer(pkg, synth, dev, E, H, I, 1, 4, seed=41, T=6)
    layer = pkg.MoeLayer(L["router"], L["bias"], L["gate"], L["up"], L["down"], 1, 4)
    outs = []
    for t in range(6):
        outs.append(layer.forward(L["x"][t:t + 1].contiguous()).clone())
    again = layer.forward(L["x"][5:6].contiguous())
    torch.cuda.synchronize()
    assert layer.status() == 0
    assert torch.equal(again, outs[5])
    for t in range(6):
        ref_y, _, _, _ = oracle_decode(orc, pkg, L, L["x"].cpu().numpy()[t])
        assert rel_l2(outs[t].cpu().numpy()[0], ref_y) < TOL


@pytest.mark.parametrize("T", [1, 40])
def test_block_forward_host_matches_device_call(pkg, synth, dev, T):
    """mmrs_moe_block_forward_host (copy in, block, copy out in one call) gives the bytes of
    mmrs_moe_block_forward on the same input."""
    import torch
    E, H, I = 32, 1024, 512
    L = make_layer(pkg, synth, dev, E, H, I, 1, 4, seed=51, T=T, x_scale=0.05)
    layer = pkg.MoeLayer(L["router"], L["bias"], L["gate"], L["up"], L["down"], 1, 4)
    x = L["x"].reshape(T, H)
    res = L["residual"].reshape(T, H)
    y_ref = layer.forward(x, residual=res)
    x_host = torch.empty(T, H, dtype=torch.float32, pin_memory=True)
    x_host.copy_(x.cpu())
    y_host = torch.zeros(T, H, dtype=torch.float32, pin_memory=True)
    x_dev = torch.empty_like(x)
    y_dev = torch.empty_like(x)
    s = torch.cuda.Stream()
    layer.forward_host(x_host, y_host, x_dev, y_dev, residual=res, stream=s)
    s.synchronize()
    assert layer.status() == 0
    assert torch.equal(y_host, y_ref.cpu())
