import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU (B200); run with -m gpu")
    config.addinivalue_line("markers", "slow: full-size cases (still a few seconds each)")


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from neuralsuite_b200 import _lib

    lib = _lib.load()  # raises if libns_b200.so is missing: no silent fallback
    assert lib.ns_device_supported() == 1, "tcgen05 kernels need an sm_100 device"
    return torch.device("cuda", torch.cuda.current_device())


@pytest.fixture(scope="session")
def port():
    import oracle

    if not os.path.exists(oracle.PORT_SO):
        oracle.build(ref=False)
    return oracle.port()
