"""Shared pytest setup: the `gpu` marker, package loading and golden data.

`-m "not gpu"` runs the oracle pins, host logic and ABI checks on any machine;
`-m gpu` runs the parity tests through the C ABI on a B200.
"""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))
TESTS = Path(__file__).resolve().parent
if str(TESTS) not in sys.path:
    sys.path.insert(0, str(TESTS))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def pkg():
    """The dispatch package, with its CUDA library built and loaded."""
    import __graft_entry__ as ge
    ge._load_build_module().build()
    mod = ge.load_package()
    mod._native.load()
    return mod


@pytest.fixture(scope="session")
def cuda_pkg(pkg):
    import torch
    if not torch.cuda.is_available():
        pytest.fail("gpu test collected on a machine without CUDA")
    major, _ = torch.cuda.get_device_capability(0)
    assert major == 10, "tests target sm_100a (B200)"
    return pkg


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as o
    return o
