"""Shared pytest setup: markers, import paths, GPU fixtures.

`-m "not gpu"` runs on a CPU-only machine; `-m gpu` needs a B200 and the built
tiny-kernel_b200/lib/libtkcuda.so (no CPU fallback exists).
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "tiny-kernel_b200")
for p in (ROOT, PKG, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 GPU and the built libtkcuda")
    config.addinivalue_line("markers", "slow: long-running CPU test")


@pytest.fixture(scope="session")
def tkdev():
    import tiny_kernel as tk
    dev = tk.init(0)
    yield dev
    dev.deinit()


@pytest.fixture(scope="session")
def tkdev_engine():
    """A second device on GPU 0 whose 1-4-row calls take the streaming engine (TK_DECODE=0, read
    when the device is created) instead of the decode kernel."""
    import tiny_kernel as tk
    old = os.environ.get("TK_DECODE")
    os.environ["TK_DECODE"] = "0"
    try:
        dev = tk.init(0)
    finally:
        if old is None:
            del os.environ["TK_DECODE"]
        else:
            os.environ["TK_DECODE"] = old
    yield dev
    dev.deinit()


@pytest.fixture(scope="session")
def torch_cuda():
    import torch
    assert torch.cuda.is_available(), "GPU test needs CUDA"
    torch.cuda.init()
    return torch
