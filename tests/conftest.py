import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))
if str(ROOT / "tests") not in sys.path:
    sys.path.insert(0, str(ROOT / "tests"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running")


@pytest.fixture(scope="session")
def spx_built():
    """Builds libspx.so in-tree if it is missing or stale (nvcc cross-compiles)."""
    from spirv_inference_b200 import build
    return build.build()


@pytest.fixture(scope="session")
def oracle_built():
    from oracle import oracle
    if not oracle.LIB_PATH.exists():
        oracle.build()
    return oracle


@pytest.fixture(scope="session")
def gpu(spx_built):
    """Device ordinal 0; GPU tests fail loudly (not skip) without a device."""
    from spirv_inference_b200.graph import device_count
    n = device_count()
    assert n > 0, "gpu-marked test needs a CUDA device"
    return 0
