import os
import sys

import pytest

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
for p in (ROOT, os.path.join(ROOT, "tests"), os.path.join(ROOT, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (the sm_100a kernels)")


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import oracle as get

    return get()


@pytest.fixture(scope="session")
def cuda_ok():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")
    return True
