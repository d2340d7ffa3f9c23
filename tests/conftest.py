"""Test configuration: markers, import paths and shared fixtures.

`gpu` tests need a B200 and call the CUDA library through its C ABI; everything else
runs on the CPU (oracle, host logic, ABI symbol checks, multi-process gloo tests).
"""
import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "llama.rs_b200")
for p in (PKG, os.path.join(REPO, "oracle"), REPO):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); calls the CUDA library")


@pytest.fixture(scope="session")
def oracle():
    import oracle as O
    O.build()
    return O


@pytest.fixture(scope="session")
def built_lib():
    from lrs import build
    build.build()
    return build.LIB


def have_gpu() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False
