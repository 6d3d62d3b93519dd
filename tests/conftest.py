"""Test configuration: the `gpu` marker and import paths.

CPU tests (``-m "not gpu"``) check the oracle against the reference's golden
vectors, the host logic against the oracle, and the C ABI's exports.  GPU
tests (``-m gpu``) run the CUDA kernels through the C ABI and compare them
with the oracle.
"""

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "cuda-kv-persistence_b200"
for p in (ROOT, PKG):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
