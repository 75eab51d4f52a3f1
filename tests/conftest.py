"""pytest configuration: the `gpu` marker, import paths, shared fixtures."""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
for p in (ROOT, ROOT / "ndtensors-rs_b200", ROOT / "tests"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); runs through the C ABI on the GPU")


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as o

    o.lib()
    return o


@pytest.fixture(scope="session")
def ndt():
    import ndtensors_b200

    ndtensors_b200.get_lib()
    return ndtensors_b200


@pytest.fixture(scope="session")
def gpu(ndt):
    """Skip-free guard: a `gpu` test must really have a device; fail loudly otherwise."""
    if not ndt.device_available():
        pytest.fail("gpu test run without a visible CUDA device")
    return ndt
