import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA sm_100 device (B200)")
    config.addinivalue_line("markers", "slow: long-running CPU test")


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


@pytest.fixture(params=["mma", "tc"])
def both_kernels(request, monkeypatch):
    """Runs a test on the mma.sync kernel and on the tcgen05 variant (PGQA_TC, read by the
    library on every call; shapes the variant does not cover stay on mma.sync)."""
    monkeypatch.setenv("PGQA_TC", "1" if request.param == "tc" else "0")
    return request.param
