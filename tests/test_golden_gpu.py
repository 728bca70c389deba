"""The CUDA path against the reference's own kernels (golden vectors, tests/golden/README.md)."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
import golden_cases as G  # noqa: E402

pytestmark = pytest.mark.gpu
GOLD = np.load(Path(__file__).resolve().parent / "golden" / "ref_kernels.npz")


def test_decode_topk_bit_exact_vs_reference(pkg, dev):
    import torch
    lg, bias = G.topk_inputs()
    b = torch.from_numpy(bias).to(dev)
    s = torch.cuda.current_stream().cuda_stream
    for i in range(lg.shape[0]):
        l = torch.from_numpy(lg[i]).to(dev)
        t = [torch.empty(8, dtype=torch.int32, device=dev) for _ in range(4)]
        pkg.lib().minimax_moe_decode_topk(l.data_ptr(), b.data_ptr(), *[x.data_ptr() for x in t], s)
        assert pkg.last_error() == 0
        got = [x.cpu().numpy() for x in t]
        assert np.array_equal(got[0].view(np.uint32), GOLD["topk_ids"][i])
        assert np.array_equal(got[1].view(np.uint32), GOLD["topk_w"][i].view(np.uint32))  # same expf: bit-exact
        assert np.array_equal(got[2].view(np.uint32), GOLD["topk_experts"][i])
        assert np.array_equal(got[3].view(np.uint32), GOLD["topk_routes"][i])


@pytest.mark.parametrize("c", G.DECODE_CASES, ids=lambda c: c["name"])
def test_decode_silu_vs_reference(pkg, dev, c):
    import torch
    L = G.layer(c)
    routes, experts, w = G.decode_routing(c)
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)  # noqa: E731
    keep = [d(G.token(c)), d(L["gate"]), d(L["up"]), d(L["down"]), d(routes), d(experts), d(w)]
    y = torch.zeros(c["H"], dtype=torch.float32, device=dev)
    pkg.lib().moe_gemm_gguf_decode_silu(*[t.data_ptr() for t in keep], y.data_ptr(), c["E"], 8, c["H"], c["I"],
                                        c["gu"], c["dn"], torch.cuda.current_stream().cuda_stream)
    assert pkg.last_error() == 0
    ref = GOLD[f"decode_{c['name']}"]
    got = y.cpu().numpy()
    assert np.linalg.norm(got - ref) / np.linalg.norm(ref) < 1e-5
