"""pytest configuration: the `gpu` marker, import paths and shared fixtures.

`-m "not gpu"` runs on any machine (oracle pinning, host logic, C-ABI loading);
`-m gpu` needs a B200 and calls libkd_attn through its C ABI.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "kandinsky.cpp_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")


@pytest.fixture(scope="session")
def kd():
    """The kd_attn package (loads libkd_attn.so, building it first if it is stale)."""
    import build  # kandinsky.cpp_b200/build.py
    build.build()
    import kd_attn
    return kd_attn


@pytest.fixture(scope="session")
def ctx(kd):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    c = kd.Context(device=0)
    yield c
    c.close()
