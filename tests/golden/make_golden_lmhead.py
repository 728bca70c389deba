"""Generates tests/golden/ref_lmhead.npz by running the reference's own Q6_K matvec kernel.

The kernel (launch_mmvq_gguf_q6_k_f32_plain with the activation quantised by
launch_mmvq_gguf_quantize_q8_1_f32, mmvq_gguf.cu:609-632, 808-809, 1296-1307) is compiled from the
reference sources, where they lie, into oracle/_ref/libref_attn.so by oracle/build_ref.sh.  Needs
a CUDA GPU (run it on the B200 box):

    python tests/golden/make_golden_lmhead.py

Inputs are regenerated from seeds (golden_cases.py), so the fixture stores only the reference
outputs.  tests/test_golden_lmhead.py checks the CPU oracle against it.
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
    lib = C.CDLL(str(ROOT / "oracle" / "_ref" / "libref_attn.so"))
    dev = torch.device("cuda:0")
    s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    x, w = G.lm_inputs()
    kpad = (G.LM_K + 511) // 512 * 512
    xd = torch.from_numpy(x).to(dev)
    wd = torch.from_numpy(np.ascontiguousarray(w)).to(dev)
    vy = torch.zeros(kpad // 32 * 36, dtype=torch.uint8, device=dev)
    y = torch.zeros(G.LM_ROWS, dtype=torch.float32, device=dev)
    P = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    lib.launch_mmvq_gguf_quantize_q8_1_f32(P(xd), P(vy), C.c_int(G.LM_K), C.c_int(kpad), C.c_int(1), s)
    lib.launch_mmvq_gguf_q6_k_f32_plain(P(wd), P(vy), P(y), C.c_int(G.LM_K), C.c_int(G.LM_ROWS),
                                        C.c_int(kpad // 32), C.c_int(G.LM_ROWS), C.c_int(1), s)
    torch.cuda.synchronize()
    out = {"logits": y.cpu().numpy(), "vy": vy.cpu().numpy()}
    np.savez_compressed(Path(__file__).resolve().parent / "ref_lmhead.npz", **out)
    print({k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
