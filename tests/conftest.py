"""Test configuration: the ``gpu`` marker, the in-tree builds, and the rule of
the reference's GPU tests (`backend/cuda/tests/cuda_tests.rs:15-28`): skip when
there is no device, fail on any other set-up error."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs through libtopos_b200.so)")


@pytest.fixture(scope="session")
def built():
    from poorgrad_b200 import build
    import oracle
    build.build()
    oracle.build()
    return True


@pytest.fixture(scope="session")
def device(built):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from poorgrad_b200 import backend
    code, message = backend.status()
    assert code == 0, f"backend status {code}: {message}"
    return True
