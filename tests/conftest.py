"""Test configuration: registers the `gpu` marker and puts the package and the
oracle on sys.path.  CPU tests (-m "not gpu") cover the oracle, the golden
fixtures, host logic and the C-ABI exports; GPU tests compare the CUDA path,
called through the C ABI, against the oracle."""
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "obsidian-memory-transformer_b200"
for p in (str(ROOT), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def orc():
    from oracle import oracle
    oracle.lib()
    return oracle


@pytest.fixture(scope="session")
def ltm():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")
    import ltm_b200
    ltm_b200.lib()
    return ltm_b200
