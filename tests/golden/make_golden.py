"""Generates tests/golden/ref_kernels.npz by running the reference's own CUDA kernels.

The kernels are compiled from the reference sources, where they lie, into oracle/_ref/libref_moe.so
by oracle/build_ref.sh.  This script needs a CUDA GPU (run it on the B200 box):

    python tests/golden/make_golden.py

Inputs are regenerated from seeds by minimax-rs_b200/synth.py, so the fixture stores only the
case parameters and the reference outputs.  tests/test_golden.py checks the CPU oracle against it.
"""
from __future__ import annotations

import ctypes as C
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(Path(__file__).resolve().parent))
import golden_cases as G  # noqa: E402


def main():
    import torch
    lib = C.CDLL(str(ROOT / "oracle" / "_ref" / "libref_moe.so"))
    dev = torch.device("cuda:0")
    s = torch.cuda.current_stream().cuda_stream
    out = {}
    P = C.c_void_p

    def d(a):
        return torch.from_numpy(np.ascontiguousarray(a)).to(dev)

    # 1. f32 dequantisation (quantized.cu:935-1004)
    for name, gt in (("q4k", G.Q4K), ("q5k", G.Q5K)):
        blocks = G.dequant_blocks(gt)
        b = d(blocks)
        y = torch.empty(blocks.shape[0] * 256, dtype=torch.float32, device=dev)
        fn = lib.ref_dequant_q4k_f32 if gt == G.Q4K else lib.ref_dequant_q5k_f32
        assert fn(P(b.data_ptr()), P(y.data_ptr()), C.c_int(blocks.shape[0]), P(s)) == 0
        out[f"dequant_{name}"] = y.cpu().numpy()

    # 2. Q8_1 quantisation (gguf.cuh:1234-1261)
    for kx in G.QUANT_K:
        x = G.quant_input(kx)
        kpad = (kx + 511) // 512 * 512
        xb = d(x)
        q = torch.zeros(x.shape[0] * kpad // 32 * 36, dtype=torch.uint8, device=dev)
        assert lib.ref_quantize_q8_1(P(xb.data_ptr()), P(q.data_ptr()), C.c_int(x.shape[0]), C.c_int(kx),
                                     C.c_int(kpad), P(s)) == 0
        out[f"q81_k{kx}"] = q.cpu().numpy()

    # 3. MMQ DS4 Q8_1 quantisation with route gather (mmq_quantize.cu:11-107, 151-160)
    x, ids, kx, div = G.mmq_quant_case()
    kpad = (kx + 511) // 512 * 512
    rows = ids.shape[0]
    xb, ib = d(x), d(ids)
    vy = torch.zeros(rows * (kpad // 128) * 144, dtype=torch.uint8, device=dev)
    lib.launch_mmq_quantize_q8_1_moe_DS4(P(xb.data_ptr()), P(ib.data_ptr()), C.c_int(div), P(vy.data_ptr()),
                                         C.c_int64(kx), C.c_int64(kx), C.c_int64(kpad), C.c_int64(rows), P(s))
    out["mmq_q81"] = vy.cpu().numpy()

    # 4. decode top-k routing (moe_gguf.cu:34-100)
    lg, bias = G.topk_inputs()
    ids_o, w_o, e_o, r_o = [], [], [], []
    bb = d(bias)
    for i in range(lg.shape[0]):
        l = d(lg[i])
        t = [torch.empty(8, dtype=torch.int32, device=dev) for _ in range(4)]
        lib.minimax_moe_decode_topk(P(l.data_ptr()), P(bb.data_ptr()), P(t[0].data_ptr()), P(t[1].data_ptr()),
                                    P(t[2].data_ptr()), P(t[3].data_ptr()), P(s))
        torch.cuda.synchronize()
        ids_o.append(t[0].cpu().numpy().view(np.uint32))
        w_o.append(t[1].cpu().numpy().view(np.float32))
        e_o.append(t[2].cpu().numpy().view(np.uint32))
        r_o.append(t[3].cpu().numpy().view(np.uint32))
    out["topk_ids"], out["topk_w"] = np.stack(ids_o), np.stack(w_o)
    out["topk_experts"], out["topk_routes"] = np.stack(e_o), np.stack(r_o)

    # 5. fused decode MoE (moe_gguf.cu:426-567)
    for c in G.DECODE_CASES:
        L = G.layer(c)
        x = G.token(c)
        routes, experts, w = G.decode_routing(c)
        y = torch.zeros(c["H"], dtype=torch.float32, device=dev)
        keep = [d(x), d(L["gate"]), d(L["up"]), d(L["down"]), d(routes), d(experts), d(w)]
        lib.moe_gemm_gguf_decode_silu(*[P(t.data_ptr()) for t in keep], P(y.data_ptr()), C.c_int(c["E"]), C.c_int(8),
                                      C.c_int(c["H"]), C.c_int(c["I"]), C.c_int(c["gu"]), C.c_int(c["dn"]), P(s))
        torch.cuda.synchronize()
        out[f"decode_{c['name']}"] = y.cpu().numpy()

    # 6/7. generic (moe_gemm_gguf) and MMQ (moe_gemm_mmq_gguf) expert GEMMs on sorted routes
    for c in G.GEMM_CASES:
        inp, w, sorted_ids, experts, tw = G.gemm_inputs(c)
        yb = torch.zeros(c["M"] * c["N"], dtype=torch.float32, device=dev)
        keep = [d(inp), d(w), d(sorted_ids), d(experts)]
        twb = d(tw) if tw is not None else None
        fn = lib.moe_gemm_mmq_gguf if c["mmq"] else lib.moe_gemm_gguf
        fn(P(keep[0].data_ptr()), P(keep[1].data_ptr()), P(keep[2].data_ptr()), P(keep[3].data_ptr()),
           P(twb.data_ptr()) if twb is not None else None, P(yb.data_ptr()), C.c_int(c["E"]), C.c_int(8),
           C.c_int(c["M"]), C.c_int(c["N"]), C.c_int(c["K"]), C.c_int(c["type"]), P(s))
        torch.cuda.synchronize()
        out[f"gemm_{c['name']}"] = yb.cpu().numpy()

    # 8. stable route sort (moe_sort.cu:21-51)
    e = G.sort_input()
    eb = d(e)
    se = torch.zeros(e.size, dtype=torch.int32, device=dev)
    sr = torch.zeros(e.size, dtype=torch.int32, device=dev)
    lib.moe_sort_routes(P(eb.data_ptr()), P(se.data_ptr()), P(sr.data_ptr()), C.c_int(e.size), C.c_int(8), P(s))
    torch.cuda.synchronize()
    out["sort_experts"], out["sort_routes"] = se.cpu().numpy().view(np.uint32), sr.cpu().numpy().view(np.uint32)

    dst = Path(__file__).resolve().parent / "ref_kernels.npz"
    np.savez_compressed(dst, **out)
    print(f"wrote {dst} ({dst.stat().st_size} bytes, {len(out)} arrays)")


if __name__ == "__main__":
    main()
