"""pytest configuration: the `gpu` marker and shared helpers.

`-m "not gpu"` runs on a CPU-only machine: oracle pins, host-side logic,
C-ABI symbol checks.  `-m gpu` runs the CUDA parity tests through the C ABI
on a B200 and fails loudly when the GPU or the built library is missing.
"""
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
for p in (str(ROOT), str(ROOT / "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) and the built libtfcuda.so")


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    from edgeexpert_b200 import _lib
    _lib.lib()  # raises if libtfcuda.so is missing: no fallback
    return torch.device("cuda:0")
