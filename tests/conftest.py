"""Shared test setup.

Markers: ``gpu`` tests need a B200 (they call libhsb.so through its C ABI);
everything else runs on the CPU.  The oracle (oracle/_build) is built on
demand; the reference bridge (oracle/_ref) exists only where it was compiled
from the reference sources.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (str(ROOT), str(ROOT / "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA sm_100 device (run with -m gpu)")


@pytest.fixture(scope="session")
def ob():
    from oracle import binding

    if not binding.ORACLE_SO.exists():
        binding.build()
    binding.oracle()
    return binding


@pytest.fixture(scope="session")
def golden():
    def load(name: str):
        return np.load(GOLDEN / name, allow_pickle=False)

    return load


@pytest.fixture(scope="session")
def cuda():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import hillserve_b200 as hsb
    from hillserve_b200 import _capi

    _capi.lib()  # fails loudly when libhsb.so is missing
    return hsb


def dev_u16(arr: np.ndarray, device="cuda"):
    import torch

    return torch.from_numpy(np.ascontiguousarray(arr).view(np.int16)).to(device)


def host_u16(t) -> np.ndarray:
    return t.detach().cpu().numpy().view(np.uint16)
