"""Shared test set-up.

Markers: ``gpu`` -- needs an sm_100 GPU; run with ``pytest -m gpu`` on a B200
box. Everything else runs on the CPU (``pytest -m "not gpu"``).

GPU tests get the library through the ``nncu`` fixture, which builds
``libnncu.so`` if it is missing and FAILS (does not skip) when no sm_100
device answers: there is no CPU fallback to pass on silently.
"""
from __future__ import annotations

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU")


@pytest.fixture(scope="session")
def nncu():
    import libllmcpu_b200 as N
    from libllmcpu_b200 import build

    if not os.path.exists(N.LIB_PATH):
        build.build()
    L = N.lib()
    rc = L.nncu_device_check(0)
    if rc != 0:
        pytest.fail(f"no usable sm_100 device: {L.nncu_last_error().decode()}")
    return N


@pytest.fixture(scope="session")
def torch_cuda(nncu):
    import torch

    assert torch.cuda.is_available()
    return torch
