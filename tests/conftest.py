"""pytest configuration: the `gpu` marker and import paths.

Tests marked `gpu` need a CUDA device (B200, sm_100a) and call the CUDA
library through its C ABI; everything else runs on the CPU.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "open-cuda_b200"), os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); calls the C ABI")


@pytest.fixture(scope="session")
def oracle():
    import oracle as _o
    _o.lib()
    return _o
