"""Shared pytest setup.

`-m "not gpu"` runs on a CPU-only machine: the oracle against the golden
fixtures, the host-side block-table logic, and loading libpagedkv.so with
every symbol include/pagedkv.h declares.  `-m gpu` runs the CUDA parity
tests; they call the kernels through the C ABI and compare with the oracle.
"""
import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
PKG = REPO / "my-inference-engine_b200"
GOLDEN = Path(__file__).resolve().parent / "golden"
for p in (str(REPO), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden():
    return GOLDEN


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("test marked gpu but CUDA is unavailable")
    import pagedkv_build

    pagedkv_build.build()  # no-op when the in-tree library is current
    import pagedkv

    pagedkv.lib()
    return torch.device("cuda", 0)
