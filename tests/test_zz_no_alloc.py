"""The allocation-free single-token entry point (mmrs_moe_block_decode_static).

It serves callers that cannot allocate device memory when they run the MoE block (an engine whose
device memory is pre-reserved by its own allocator, or a call site with no workspace to pass);
its scratch is a fixed device array inside the library.  This file is collected last so a run
that stops at the first failure has already run every other test."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from conftest import rel_l2
from moe_cases import make_layer

pytestmark = pytest.mark.gpu

TOL = 1e-3  # same relative-L2 bound as the other MoE block tests


def test_static_scratch_entry_matches_workspace_entry(pkg, synth, dev):
    import torch
    L = make_layer(pkg, synth, dev, 256, 3072, 1536, pkg.Q4K, pkg.Q5K, seed=77, T=2)
    layer = pkg.MoeLayer(L["router"], L["bias"], L["gate"], L["up"], L["down"], pkg.Q4K, pkg.Q5K)
    stream = torch.cuda.current_stream().cuda_stream
    for t in range(2):  # two calls in a row share (and reuse) the fixed scratch
        x, res = L["x"][t:t + 1].contiguous(), L["residual"][t:t + 1].contiguous()
        ids_ref = torch.empty(1, 8, dtype=torch.int32, device=dev)
        w_ref = torch.empty(1, 8, dtype=torch.float32, device=dev)
        y_ref = layer.forward(x, residual=res, topk_ids=ids_ref, topk_w=w_ref)
        y = torch.empty_like(x)
        ids = torch.empty(1, 8, dtype=torch.int32, device=dev)
        w = torch.empty(1, 8, dtype=torch.float32, device=dev)
        rc = pkg.lib().mmrs_moe_block_decode_static(C.byref(layer.c), x.data_ptr(), res.data_ptr(), y.data_ptr(),
                                                     ids.data_ptr(), w.data_ptr(), stream)
        assert rc == pkg.MMRS_OK
        # the static call's own status word (in the library's fixed array), read before the next call
        assert pkg.lib().mmrs_moe_static_status(stream) == pkg.MMRS_OK
        assert layer.status() == 0
        assert torch.equal(ids, ids_ref)
        np.testing.assert_allclose(w.cpu().numpy(), w_ref.cpu().numpy(), rtol=1e-6)
        assert rel_l2(y.cpu().numpy(), y_ref.cpu().numpy()) < TOL


def test_static_scratch_entry_rejects_oversized_problems(pkg, dev):
    import torch
    z = torch.zeros(16, dtype=torch.uint8, device=dev)
    big = pkg.MmrsMoeWeights(z.data_ptr(), z.data_ptr(), z.data_ptr(), z.data_ptr(), z.data_ptr(), pkg.Q4K,
                             pkg.Q5K, 256, 8, 3072, 3072)  # inter 3072 > 1536
    x = torch.zeros(1, 3072, dtype=torch.float32, device=dev)
    rc = pkg.lib().mmrs_moe_block_decode_static(C.byref(big), x.data_ptr(), None, x.data_ptr(), None, None,
                                                 torch.cuda.current_stream().cuda_stream)
    assert rc == pkg.MMRS_ERR_SCRATCH_LIMIT
