"""Shared pytest configuration.

Markers: ``gpu`` marks tests that need a B200 (sm_100).  They call the product
through the C ABI of ``libkatab200.so`` and compare against the CPU oracle.
"""

import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU (run with -m gpu)")


@pytest.fixture(scope="session")
def cuda():
    """The torch CUDA module on a checked sm_100 device (allocator/streams only)."""
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from rust_katago_b200 import _capi

    _capi.call("kb_device_check", torch.cuda.current_device())
    return torch


@pytest.fixture(scope="session")
def oracle():
    import oracle as o

    o.build()
    return o
