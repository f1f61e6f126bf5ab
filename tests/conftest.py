"""pytest configuration: the `gpu` marker and import paths.

Tests marked ``gpu`` need a B200 and the built CUDA library; everything else
runs on CPU (oracle against golden vectors, host logic, ABI symbol checks).
"""
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "lanczos-gpu_b200"
for p in (str(ROOT), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)

os.environ.setdefault("OMP_NUM_THREADS", str(os.cpu_count() or 1))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built sm_100a library")


@pytest.fixture(scope="session")
def golden_dir():
    return ROOT / "tests" / "golden"
