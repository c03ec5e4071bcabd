import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a) and the built library")
    config.addinivalue_line("markers", "slow: full-size parity runs (minutes)")


@pytest.fixture(scope="session")
def oracle_lib():
    import oracle

    oracle.build()
    return oracle


@pytest.fixture(scope="session")
def cuda_lib():
    """The built libqwenscriber_cuda.so (built on demand, as __graft_entry__.build does)."""
    from qwenscriber_b200 import build, runtime

    if not os.path.exists(runtime.LIB_PATH):
        build.build()
    return runtime.lib()


@pytest.fixture(scope="session")
def gpu():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but no CUDA device is visible")
    return torch.device("cuda:0")
