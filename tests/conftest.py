"""Shared test set-up: the `gpu` marker, import paths, and builds.

`-m "not gpu"` covers the oracle (pinned against the reference's own C code and
the committed golden fixtures), host logic and the C-ABI exports; `-m gpu`
runs the CUDA path through the C ABI against the oracle.
"""
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "esp32-needle-3_b200")
ORACLE = os.path.join(ROOT, "oracle")
for p in (PKG, ORACLE, ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU (runs the CUDA path)")


def _make(path):
    subprocess.run(["make", "-s", "-C", path], check=True)


@pytest.fixture(scope="session", autouse=True)
def built():
    """Builds the oracle and the library if a tree arrives without them."""
    if not os.path.exists(os.path.join(ORACLE, "libndoracle.so")):
        _make(ORACLE)
    if not os.path.exists(os.path.join(PKG, "libndattn.so")):
        _make(PKG)
    yield


@pytest.fixture(scope="session")
def has_gpu():
    import torch
    return torch.cuda.is_available() and torch.cuda.get_device_capability(0)[0] == 10


@pytest.fixture(autouse=True)
def _gpu_gate(request, has_gpu):
    if request.node.get_closest_marker("gpu") and not has_gpu:
        pytest.skip("needs an sm_100 GPU")
