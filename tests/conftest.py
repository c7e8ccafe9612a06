"""Shared fixtures.  GPU tests are marked `gpu`; everything else runs on the CPU."""
import importlib
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

PKG_NAME = "gemma-webgpu-engine_b200"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def load_pkg():
    return importlib.import_module(PKG_NAME)


@pytest.fixture(scope="session")
def pkg():
    return load_pkg()


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O
    O.lib()
    return O


@pytest.fixture(scope="session")
def sampler(pkg):
    import torch
    assert torch.cuda.is_available(), "gpu tests need a CUDA device"
    s = pkg.GpuSampler(0)
    yield s
    s.close()
