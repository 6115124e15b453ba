import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")
    # Build the native library and the oracle in-tree if they are missing or
    # stale (make is incremental).
    from cuda_micro_bench_b200 import build as _build
    _build.build()
    import oracle
    oracle.build()


@pytest.fixture(scope="session")
def cmb():
    import cuda_micro_bench_b200 as c
    return c


@pytest.fixture(scope="session")
def orc():
    import oracle
    return oracle.load()


@pytest.fixture(scope="session")
def cuda():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    major, minor = torch.cuda.get_device_capability(0)
    assert major == 10, f"GPU tests need sm_100 (got sm_{major}{minor})"
    torch.cuda.set_device(0)
    return torch
