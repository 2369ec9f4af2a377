import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built libcvhrf.so")


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


@pytest.fixture(scope="session")
def ref():
    """The reference's own kernels (oracle/_ref), or skip if they were not built."""
    from oracle import ref_harness
    if not ref_harness.available():
        pytest.skip("reference kernels not built (python oracle/build_ref.py)")
    return ref_harness
