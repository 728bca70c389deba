"""Seeded MoE-layer builders shared by the GPU tests (inputs generated on the device by the
package's synthetic generator; the oracle receives copies of exactly the same bytes)."""
from __future__ import annotations

import numpy as np


def make_layer(pkg, synth, dev, E, H, I, gu_type, dn_type, seed, layer=0, T=1, x_bf16=True, zipf=False,
               x_scale=1.0):
    import torch
    st = synth.layer_streams(layer)
    x = torch.empty(T * H, dtype=torch.float32, device=dev)
    pkg.synth_normal(x, seed, st["x"], x_scale, bf16=x_bf16)
    router = torch.empty(E * H, dtype=torch.float32, device=dev)
    pkg.synth_normal(router, seed, st["router"], 0.02)
    if zipf:
        bias = torch.from_numpy(synth.zipf_bias(E, seed)).to(dev)
    else:
        bias = torch.empty(E, dtype=torch.float32, device=dev)
        pkg.synth_normal(bias, seed, st["bias"], 0.01)
    residual = torch.empty(T * H, dtype=torch.float32, device=dev)
    pkg.synth_normal(residual, seed, st["residual"], 1.0)
    gate = torch.empty(E * I * pkg.row_bytes(gu_type, H), dtype=torch.uint8, device=dev)
    up = torch.empty_like(gate)
    down = torch.empty(E * H * pkg.row_bytes(dn_type, I), dtype=torch.uint8, device=dev)
    pkg.synth_kquant(gate, gu_type, seed, st["gate"], E, I, H)
    pkg.synth_kquant(up, gu_type, seed, st["up"], E, I, H)
    pkg.synth_kquant(down, dn_type, seed, st["down"], E, H, I)
    return dict(x=x.view(T, H), router=router.view(E, H), bias=bias, residual=residual.view(T, H), gate=gate,
                up=up, down=down, E=E, H=H, I=I, gu_type=gu_type, dn_type=dn_type)


def expert_slices(pkg, L, experts):
    """Host copies of the given experts' gate/up/down bytes, stacked in the given order."""
    E, H, I = L["E"], L["H"], L["I"]
    gsz = I * pkg.row_bytes(L["gu_type"], H)
    dsz = H * pkg.row_bytes(L["dn_type"], I)
    g = L["gate"].view(E, gsz)[list(experts)].cpu().numpy()
    u = L["up"].view(E, gsz)[list(experts)].cpu().numpy()
    d = L["down"].view(E, dsz)[list(experts)].cpu().numpy()
    return g, u, d


def oracle_decode(orc, pkg, L, x_row, residual_row=None):
    """Oracle of the single-token block: canonical router logits, decode top-8 and the decode
    dataflow of moe_gemm_gguf_decode_silu on the 8 selected experts (gathered to the host)."""
    router = L["router"].cpu().numpy()
    bias = L["bias"].cpu().numpy()
    logits = orc.router_logits(x_row.reshape(1, -1), router)[0]
    ids, w, eids, rids = orc.decode_topk(logits, bias) if L["E"] == 256 else _generic_topk(orc, logits, bias)
    g, u, d = expert_slices(pkg, L, eids)
    y = orc.moe_decode_silu(x_row, g, u, d, rids.astype(np.int32), np.arange(8, dtype=np.int32), w, 8,
                            L["H"], L["I"], L["gu_type"], L["dn_type"])
    if residual_row is not None:
        y = (y + residual_row).astype(np.float32)
    return y, ids, w, logits


def _generic_topk(orc, logits, bias):
    ids, w = orc.route_topk(logits.reshape(1, -1), bias)
    ids, w = ids[0], w[0]
    order = np.argsort(ids, kind="stable")
    return ids, w, ids[order], order.astype(np.uint32)
