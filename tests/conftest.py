"""Shared pytest setup: import paths, the gpu marker, GPU/oracle fixtures."""
from __future__ import annotations

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "cosyvoice.cpp_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O
    O.build()
    return O


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test collected without a CUDA device")
    return torch


@pytest.fixture(scope="session")
def cv(cuda):
    import cvattn
    return cvattn


@pytest.fixture(scope="session")
def ctx(cv):
    c = cv.Context(0)
    yield c
    c.close()


@pytest.fixture(autouse=True)
def _check_device_status(request):
    """After every GPU test the context's status word must be clean unless the test consumed it."""
    yield
    if "gpu" in request.keywords and "ctx" in request.fixturenames:
        c = request.getfixturevalue("ctx")
        st, detail = c.sync_status()
        assert st == 0, f"device status word left set (detail {detail})"
