"""Generates tests/golden/ref_attn.npz by running the reference's own decode-attention kernels.

The kernels are compiled from the reference sources, where they lie, into oracle/_ref/libref_attn.so
by oracle/build_ref.sh (mmvq_gguf.cu, decode_attention.cu).  Needs a CUDA GPU (run it on the B200
box):

    python tests/golden/make_golden_attn.py

Inputs are regenerated from seeds (golden_cases.py), so the fixture stores only the reference
outputs.  tests/test_golden_attn.py checks the CPU oracle against it.
"""
from __future__ import annotations

import ctypes as C
import math
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(Path(__file__).resolve().parent))
import golden_cases as G  # noqa: E402


def main():
    import torch
    lib = C.CDLL(str(ROOT / "oracle" / "_ref" / "libref_attn.so"))
    dev = torch.device("cuda:0")
    s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    P = C.c_void_p
    out = {}

    def d(a):
        return torch.from_numpy(np.ascontiguousarray(a)).to(dev)

    def ptr(t):
        return P(t.data_ptr())

    # 1. Q8_0 QKV projection + Q/K RMSNorm + f16 (mmvq_gguf.cu:814-885, 1309-1336)
    x, wq, wk, wv, qa, ka = G.qkv_inputs()
    kpad = (G.ATTN_H + 511) // 512 * 512
    n = G.Q_ROWS + G.K_ROWS + G.V_ROWS
    keep = [d(x), d(wq), d(wk), d(wv), d(qa), d(ka)]
    vy = torch.zeros(kpad // 32 * 36, dtype=torch.uint8, device=dev)
    proj = torch.zeros(n, dtype=torch.float32, device=dev)
    dst = torch.zeros(n, dtype=torch.float16, device=dev)
    lib.launch_mmvq_gguf_qkv_q8_0_f32_rmsnorm_f16(
        ptr(keep[0]), ptr(vy), ptr(keep[1]), ptr(keep[2]), ptr(keep[3]), ptr(proj), ptr(keep[4]), ptr(keep[5]),
        ptr(dst), C.c_int(G.ATTN_H), C.c_int(kpad), C.c_int(G.Q_ROWS), C.c_int(G.K_ROWS), C.c_int(G.V_ROWS),
        C.c_float(1e-6), s)
    torch.cuda.synchronize()
    out["qkv_proj"] = proj.cpu().numpy()
    out["qkv_f16"] = dst.cpu().numpy().view(np.uint16)

    # 2. partial RoPE on f16 Q and K (mmvq_gguf.cu:1038-1066)
    q, k, cos, sin = G.rope_inputs()
    qd, kd, cd, sd = d(q), d(k), d(cos), d(sin)
    for pos in G.ROPE_POS:
        r = torch.zeros(G.Q_ROWS + G.K_ROWS, dtype=torch.float16, device=dev)
        lib.launch_partial_rope_f16(ptr(qd), ptr(kd), ptr(cd), ptr(sd), ptr(r), C.c_int(G.Q_ROWS), C.c_int(G.K_ROWS),
                                    C.c_int(G.HD), C.c_int(G.ROT), C.c_int(pos), s)
        torch.cuda.synchronize()
        out[f"rope_p{pos}"] = r.cpu().numpy().view(np.uint16)

    # 3. split-K GQA decode + combine (decode_attention.cu:311-843)
    scale = 1.0 / math.sqrt(G.HD)
    for seq_len, splits in G.GQA_CASES:
        qh, kh, vh = G.gqa_inputs(seq_len)
        qd, kd, vd = d(qh), d(kh), d(vh)
        part = torch.zeros(splits * G.QH * (G.HD + 2), dtype=torch.float32, device=dev)
        o = torch.zeros(G.QH * G.HD, dtype=torch.float16, device=dev)
        lib.launch_gqa_decode_mma_f16_128(ptr(qd), ptr(kd), ptr(vd), ptr(part), ptr(o), C.c_int(seq_len),
                                          C.c_int(G.HD), C.c_int(G.KV_CAP * G.HD), C.c_int(G.KV_CAP * G.HD),
                                          C.c_int(splits), C.c_int(G.QH), C.c_int(G.KVH), C.c_float(scale),
                                          C.c_int(0), s)
        torch.cuda.synchronize()
        out[f"gqa_s{seq_len}_n{splits}"] = o.cpu().numpy().view(np.uint16)

    # 4. output projection: Q8_1 of the f32 attention output, Q8_0 matvec (mmvq_gguf.cu:1137-1200)
    a, wo = G.oproj_inputs()
    ad, wd = d(a), d(wo)
    kpad = (G.Q_ROWS + 511) // 512 * 512
    vy = torch.zeros(kpad // 32 * 36, dtype=torch.uint8, device=dev)
    y = torch.zeros(G.ATTN_H, dtype=torch.float32, device=dev)
    lib.launch_mmvq_gguf_quantize_q8_1_f32(ptr(ad), ptr(vy), C.c_int(G.Q_ROWS), C.c_int(kpad), C.c_int(1), s)
    lib.launch_mmvq_gguf_q8_0_f32_plain(ptr(wd), ptr(vy), ptr(y), C.c_int(G.Q_ROWS), C.c_int(G.ATTN_H),
                                        C.c_int(kpad // 32), C.c_int(G.ATTN_H), C.c_int(1), s)
    torch.cuda.synchronize()
    out["oproj"] = y.cpu().numpy()

    dst_path = Path(__file__).resolve().parent / "ref_attn.npz"
    np.savez_compressed(dst_path, **out)
    print(f"wrote {dst_path} ({dst_path.stat().st_size} bytes, {len(out)} arrays)")


if __name__ == "__main__":
    main()
