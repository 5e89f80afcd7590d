"""Test configuration: the `gpu` marker, import paths, and shared helpers.

`-m "not gpu"` runs here without a GPU: the oracle against the reference's golden vectors, the oracle's
own math checks, host-side logic, and the C-ABI library's exports and argument validation (no launches).
`-m gpu` runs the CUDA path through the C ABI against the oracle.
"""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "comfyui-hy-nomas_b200")
for p in (ROOT, PKG_DIR, os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU; runs the CUDA path through the C ABI")
    config.addinivalue_line("markers", "slow: full-size (benchmark shape) property checks")


@pytest.fixture(scope="session")
def golden():
    def load(name):
        return np.load(os.path.join(GOLDEN, name + ".npz"))
    return load


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O
    O.build()
    return O


@pytest.fixture(scope="session")
def hn():
    """The product package (needs libhynomas_b200.so; built by __graft_entry__.build())."""
    from hy_nomas_b200 import build
    build.build()
    import hy_nomas_b200.fused as fused
    import hy_nomas_b200.kernels as kernels
    import hy_nomas_b200.ops as ops
    import hy_nomas_b200.world as world
    from hy_nomas_b200 import _lib

    class NS:
        pass
    ns = NS()
    ns.kernels, ns.fused, ns.ops, ns.world, ns.lib = kernels, fused, ops, world, _lib
    return ns


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, minor = torch.cuda.get_device_capability()
    if (major, minor) != (10, 0):
        pytest.skip(f"needs sm_100 (B200), found sm_{major}{minor}")
    return torch.device("cuda:0")
