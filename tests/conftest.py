"""Test configuration: the `gpu` marker and import paths.

`-m "not gpu"` runs on a CPU-only machine: oracle checks against the golden
fixtures and the numpy twin, host logic, ABI exports, and 2-rank gloo tests of
the sharded algorithm. `-m gpu` runs the parity tests of the CUDA library
(through its C ABI) against the oracle on a B200.
"""
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
PKG = ROOT / "mlx-swift-lm_b200"
for p in (str(ROOT), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a) and the built library")


@pytest.fixture(scope="session")
def oracle_lib():
    import oracle
    oracle.lib()
    return oracle


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("gpu test selected but no CUDA device is visible")
    import sparse_decode
    sparse_decode.lib()
    return torch
