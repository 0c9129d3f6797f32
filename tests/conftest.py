"""Shared test set-up: import paths, the `gpu` marker, and build-on-demand of the
CPU oracle (gcc) and of libsdq.so (nvcc cross-compiles without a GPU)."""
from __future__ import annotations

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "stable-diffusion.rs_b200")
ORACLE = os.path.join(ROOT, "oracle")
for p in (PKG, ORACLE, ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) CUDA device")


@pytest.fixture(scope="session", autouse=True)
def _built():
    import oracle as O

    O.build()
    lib = os.path.join(PKG, "libsdq.so")
    if not os.path.exists(lib):
        sys.path.insert(0, PKG)
        import build as B

        B.build()
    yield


def gpu_available() -> bool:
    try:
        import torch

        return torch.cuda.is_available() and torch.cuda.get_device_capability(0) == (10, 0)
    except Exception:
        return False
