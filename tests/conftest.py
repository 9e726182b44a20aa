"""Shared test setup: import paths, the `gpu` marker, the oracle build."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "omni.js_b200"), os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); runs the native sampler")


@pytest.fixture(scope="session")
def oracle():
    import ms_oracle

    ms_oracle.build()
    return ms_oracle


@pytest.fixture(scope="session")
def sampler():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test collected on a machine without CUDA")
    torch.cuda.init()
    from minisample import Sampler

    s = Sampler()
    yield s
    s.close()
