"""Shared fixtures.  GPU tests are marked `gpu`; everything else runs on the CPU."""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "oracle"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def pkg():
    import __graft_entry__ as ge
    lib_path = ge.PKG_DIR / "lib" / "libminimax_moe.so"
    if not lib_path.exists():
        ge.build()
    return ge.load_package()


@pytest.fixture(scope="session")
def synth():
    import __graft_entry__ as ge
    return ge.load_synth()


@pytest.fixture(scope="session")
def orc():
    import oracle
    oracle.build()
    return oracle


@pytest.fixture(scope="session")
def dev():
    import torch
    assert torch.cuda.is_available(), "GPU test on a machine without CUDA"
    return torch.device("cuda:0")


def rel_l2(got, ref) -> float:
    import numpy as np
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30))
