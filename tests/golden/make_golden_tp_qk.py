"""Generates tests/golden/ref_tp_qk.npz by running the reference's own tensor-parallel Q/K
RMSNorm kernels for both ranks of TP = 2.

launch_qkv_tp_sumsq_f32 (mmvq_gguf.cu:970-990, 1360-1366) on each rank's projection, the two
ranks' statistics summed (the all-reduce of src/tensor_parallel_model.rs:407-410), then
launch_qkv_tp_rmsnorm_rope_f16 (mmvq_gguf.cu:995-1034, 1368-1382) on each rank at each position of
golden_cases.TP_POS.  The kernels are compiled from the reference sources, where they lie, into
oracle/_ref/libref_attn.so by oracle/build_ref.sh.  Needs a CUDA GPU:

    python tests/golden/make_golden_tp_qk.py [output.npz]

Inputs are regenerated from seeds (golden_cases.py); the fixture stores only the outputs.
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


def run(lib, dev) -> dict:
    """Both ranks through `lib`'s two launchers: {'stats': [2][2], 'global': [2], 'dst_r<rank>_p<pos>'}."""
    import torch
    s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    P = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)  # noqa: E731
    out = {}
    ins = [[T(a) for a in G.tp_qk_inputs(r)] for r in range(2)]
    stats = []
    for r in range(2):
        q, k = ins[r][0], ins[r][1]
        st = torch.zeros(2, dtype=torch.float32, device=dev)
        lib.launch_qkv_tp_sumsq_f32(P(q), P(k), P(st), C.c_int(q.numel()), C.c_int(k.numel()), s)
        stats.append(st)
    torch.cuda.synchronize()
    glob = stats[0] + stats[1]
    out["stats"] = torch.stack(stats).cpu().numpy()
    out["global"] = glob.cpu().numpy()
    for r in range(2):
        q, k, v, qa, ka, cos, sin = ins[r]
        for pos in G.TP_POS:
            dst = torch.zeros(q.numel() + k.numel() + v.numel(), dtype=torch.float16, device=dev)
            lib.launch_qkv_tp_rmsnorm_rope_f16(P(q), P(k), P(v), P(glob), P(qa), P(ka), P(cos), P(sin), P(dst),
                                               C.c_int(q.numel()), C.c_int(k.numel()), C.c_int(v.numel()),
                                               C.c_int(G.TP_Q_FULL), C.c_int(G.TP_K_FULL), C.c_int(G.HD),
                                               C.c_int(G.ROT), C.c_int(pos), C.c_float(1e-6), s)
            torch.cuda.synchronize()
            out[f"dst_r{r}_p{pos}"] = dst.cpu().numpy().view(np.uint16)
    return out


def main():
    import torch
    lib = C.CDLL(str(ROOT / "oracle" / "_ref" / "libref_attn.so"))
    path = Path(sys.argv[1]) if len(sys.argv) > 1 else Path(__file__).resolve().parent / "ref_tp_qk.npz"
    np.savez_compressed(path, **run(lib, torch.device("cuda:0")))
    print(f"wrote {path}")


if __name__ == "__main__":
    main()
