import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (sm_100a B200)")
    config.addinivalue_line("markers", "multigpu: needs 2 or more CUDA GPUs")


@pytest.fixture(scope="session")
def native_lib():
    """The built C-ABI library (built here with nvcc if it is missing)."""
    from pyre_b200 import _native, build
    if not _native.LIB_PATH.exists():
        build.build()
    return _native.load()


@pytest.fixture(scope="session")
def oracle_lib():
    """ctypes handle of the oracle's C restatement (built with make if missing)."""
    from oracle import cref
    return cref.load()


def cuda_ok() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False
