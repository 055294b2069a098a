import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a); run with -m gpu")


def cuda_available() -> bool:
    import torch

    return torch.cuda.is_available()


def device_count() -> int:
    import torch

    return torch.cuda.device_count() if torch.cuda.is_available() else 0


@pytest.fixture(scope="session")
def kvx_lib():
    """The built C-ABI library (built here if missing; nvcc cross-compiles without a GPU)."""
    from lmpool_b200 import _build, _capi

    if os.environ.get("LMPOOL_B200_NO_BUILD") != "1":
        _build.build()
    return _capi.lib()


@pytest.fixture(scope="session")
def require_gpu(kvx_lib):
    if not cuda_available():
        pytest.skip("no CUDA device")
    return kvx_lib
