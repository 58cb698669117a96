"""Shared pytest setup: import paths, the `gpu` marker, seeded input helpers."""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "ltx-2_b200")
DROPIN = os.path.join(PKG, "dropin")  # blockwise_cpp, the reference's compiled-module name
for p in (DROPIN, PKG, REPO):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU; runs through the C-ABI library")


@pytest.fixture(scope="session")
def golden():
    def load(name):
        return np.load(os.path.join(GOLDEN, name))
    return load


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but no CUDA device is visible")
    from ltx_kernels import _lib
    _lib.load()  # the sm_100a library must load; no fallback exists
    return torch.device("cuda", 0)


@pytest.fixture(autouse=True)
def _device_status_clean(request):
    """After every GPU test, the kernels' bounded-wait status word must be 0."""
    yield
    if request.node.get_closest_marker("gpu") is None:
        return
    import torch
    if not torch.cuda.is_available():
        return
    from ltx_kernels.blockwise import ops
    torch.cuda.synchronize()
    assert ops.device_status(clear=True) == 0, "a kernel recorded a bounded-wait timeout"
