"""pytest configuration: the `gpu` marker, import paths and shared fixtures.

`-m "not gpu"` runs the oracle-vs-golden, host-logic and C-ABI export tests on
CPU; `-m gpu` runs the parity tests, which call the CUDA path through the C ABI
and fail (never skip silently onto another path) when CUDA is unavailable.
"""
from __future__ import annotations

import pathlib
import sys

import pytest

ROOT = pathlib.Path(__file__).resolve().parent.parent
TESTS = pathlib.Path(__file__).resolve().parent
for p in (str(ROOT), str(TESTS)):
    if p not in sys.path:
        sys.path.insert(0, p)

import __graft_entry__  # noqa: E402

__graft_entry__.load_package()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200, sm_100a) device")


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    return dict(np.load(TESTS / "golden" / "reference_golden.npz"))


@pytest.fixture(scope="session")
def cuda_dev():
    import torch
    assert torch.cuda.is_available(), "GPU test run without a CUDA device"
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    from wavefront_decoding_b200 import _abi
    _abi.load()
    return dev
