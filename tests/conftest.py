"""Test configuration: the `gpu` marker, import paths, shared fixtures.

`-m "not gpu"` runs on any machine (the oracle, the host logic, the C-ABI
library's loading and exports); `-m gpu` needs a B200 and the in-tree build.
"""
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built pantheon_b200 library")


@pytest.fixture(scope="session")
def oracle():
    from oracle import qg_oracle
    qg_oracle.lib()
    return qg_oracle


@pytest.fixture(scope="session")
def qglib():
    """The in-tree C-ABI library, built if missing (build needs only nvcc)."""
    import pantheon_b200
    from pantheon_b200 import build
    if not all(x.exists() for x in (pantheon_b200.LIB_PATH, pantheon_b200.BIN_PATH, pantheon_b200.DECODE_BIN_PATH,
                                     pantheon_b200.MMA_BIN_PATH)):
        build.build()
    return pantheon_b200.load_library()


@pytest.fixture(scope="session")
def cuda_device(qglib):
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a visible CUDA device")
    major, minor = torch.cuda.get_device_capability(0)
    if (major, minor) != (10, 0):
        pytest.fail(f"GPU tests need sm_100 (B200); found sm_{major}{minor}")
    return torch.device("cuda:0")
