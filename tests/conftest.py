"""Shared test setup: the `gpu` marker, import paths and fixtures.

Tests marked `gpu` need a B200 (sm_100a) and the built library; everything else
runs on the CPU: the oracle against the reference and its golden vectors, the C
ABI's exports and host-side logic, and the multi-process (gloo) sharding path.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU and the built CUDA library")


@pytest.fixture(scope="session")
def oracle_lib():
    from oracle import oracle
    if not oracle.available("port"):
        oracle.build()
    return oracle


@pytest.fixture(scope="session")
def fe_lib():
    from fastembed_b200 import build
    build.build()
    from fastembed_b200 import capi
    return capi.lib()


@pytest.fixture(scope="session")
def cuda_dev(fe_lib):
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a visible CUDA device")
    return torch.device("cuda", 0)
