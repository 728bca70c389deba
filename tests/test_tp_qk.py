"""Tensor-parallel Q/K RMSNorm of a decode step (TP = 2): launch_qkv_tp_sumsq_f32 and
launch_qkv_tp_rmsnorm_rope_f16 (mmvq_gguf.cu:970-1034; src/tensor_parallel_model.rs:123-168,
407-419).  CPU: the oracle against the reference kernels' recorded outputs
(tests/golden/ref_tp_qk.npz, made by tests/golden/make_golden_tp_qk.py on a B200).  GPU: the CUDA
launchers bit-identical to the same recording, and the two ranks' halves close to the
single-GPU full-width normalisation."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
import golden_cases as G  # noqa: E402

GOLD = Path(__file__).resolve().parent / "golden" / "ref_tp_qk.npz"


@pytest.fixture(scope="module")
def gold():
    if not GOLD.exists():
        pytest.fail("tests/golden/ref_tp_qk.npz missing: run tests/golden/make_golden_tp_qk.py on a GPU")
    return np.load(GOLD)


def _half_ulps(a_bits, b_bits):
    a = a_bits.view(np.float16).astype(np.float64)
    b = b_bits.view(np.float16).astype(np.float64)
    ulp = np.spacing(np.maximum(np.abs(a), np.abs(b)).astype(np.float16)).astype(np.float64)
    return np.abs(a - b) / np.maximum(ulp, 1e-12)


def test_oracle_matches_reference_recording(orc, gold):
    for r in range(2):
        q, k, v, qa, ka, cos, sin = G.tp_qk_inputs(r)
        np.testing.assert_allclose(orc.tp_qk_sumsq(q, k), gold["stats"][r], rtol=1e-5)
        for pos in G.TP_POS:
            want = gold[f"dst_r{r}_p{pos}"]
            got = orc.tp_qk_rmsnorm_rope_f16(q, k, v, gold["global"], qa, ka, cos, sin, G.TP_Q_FULL, G.TP_K_FULL,
                                             G.HD, G.ROT, pos)
            d = _half_ulps(got, want)
            assert d.max() <= 2 and (d == 0).mean() > 0.99, (r, pos, d.max(), (d == 0).mean())


@pytest.mark.gpu
def test_cuda_launchers_bit_identical_to_reference(pkg, gold, dev):
    import importlib
    mk = importlib.import_module("make_golden_tp_qk")
    got = mk.run(pkg.lib(), dev)
    assert pkg.last_error() == 0
    assert np.array_equal(got["stats"], gold["stats"]) and np.array_equal(got["global"], gold["global"])
    for r in range(2):
        for pos in G.TP_POS:
            assert np.array_equal(got[f"dst_r{r}_p{pos}"], gold[f"dst_r{r}_p{pos}"]), (r, pos)


def test_ranks_agree_with_full_width_normalisation(orc, gold):
    """Rank 0's and rank 1's Q heads, normalised with the all-reduced sums, are the full-width
    RMSNorm + RoPE of the concatenated projection (the single-GPU path), up to the statistics'
    summation order."""
    ins = [G.tp_qk_inputs(r) for r in range(2)]
    q = np.concatenate([ins[0][0], ins[1][0]])
    k = np.concatenate([ins[0][1], ins[1][1]])
    qa = np.concatenate([ins[0][3], ins[1][3]])
    ka = np.concatenate([ins[0][4], ins[1][4]])
    cos, sin = ins[0][5], ins[0][6]
    full = orc.tp_qk_rmsnorm_rope_f16(q, k, np.zeros(0, np.float32), orc.tp_qk_sumsq(q, k), qa, ka, cos, sin,
                                      G.TP_Q_FULL, G.TP_K_FULL, G.HD, G.ROT, G.TP_POS[1])
    fq, fk = full[:G.TP_Q_FULL], full[G.TP_Q_FULL:]
    for r in range(2):
        got = gold[f"dst_r{r}_p{G.TP_POS[1]}"]
        gq, gk = got[:G.TP_Q_LOCAL], got[G.TP_Q_LOCAL:G.TP_Q_LOCAL + G.TP_KV_LOCAL]
        dq = _half_ulps(gq, fq[r * G.TP_Q_LOCAL:(r + 1) * G.TP_Q_LOCAL])
        dk = _half_ulps(gk, fk[r * G.TP_KV_LOCAL:(r + 1) * G.TP_KV_LOCAL])
        assert dq.max() <= 2 and dk.max() <= 2


def _tp_rank_main(rank, world, port, q):
    """One TP rank on CPU: its rank-local statistics (the reference kernel's, from the recording),
    the two-float all-reduce over gloo (the collective of src/tensor_parallel_model.rs:407-410),
    then the normalisation with the reduced statistics (oracle)."""
    import os
    import sys
    root = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(root / "oracle"), str(root / "tests" / "golden")]
    import torch
    import torch.distributed as dist

    import golden_cases as Gc
    import oracle
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    gold = np.load(GOLD)
    stats = torch.from_numpy(np.array(gold["stats"][rank], dtype=np.float32))
    dist.all_reduce(stats)
    qq, k, v, qa, ka, cos, sin = Gc.tp_qk_inputs(rank)
    dst = oracle.tp_qk_rmsnorm_rope_f16(qq, k, v, stats.numpy(), qa, ka, cos, sin, Gc.TP_Q_FULL, Gc.TP_K_FULL,
                                        Gc.HD, Gc.ROT, Gc.TP_POS[1])
    q.put((rank, stats.numpy().tobytes(), _half_ulps(dst, gold[f"dst_r{rank}_p{Gc.TP_POS[1]}"]).max()))
    dist.destroy_process_group()


def test_tp2_statistics_all_reduce_gloo(gold):
    """world_size 2 on CPU: the all-reduced statistics equal the recorded global sums bit for bit,
    and each rank's normalisation from them matches its recorded output."""
    import socket

    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_tp_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, stats, worst in results:
        assert stats == np.asarray(gold["global"], np.float32).tobytes()
        assert worst <= 2
