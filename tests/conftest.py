"""Shared test set-up: the `gpu` marker, repo-root imports, seeded inputs."""
from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))
GOLDEN = ROOT / "tests" / "golden"

# every device-side error is surfaced right after the call in the tests
os.environ.setdefault("FLASH_MAXSIM_SYNC_CHECK", "1")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200, sm_100a) device")


def pytest_sessionstart(session):
    # the CUDA library is built in-tree (nvcc cross-compiles without a GPU)
    import importlib.util
    spec = importlib.util.spec_from_file_location("_fm_build", ROOT / "flash_maxsim_b200" / "build.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    mod.build()


def golden(name: str):
    return np.load(GOLDEN / f"{name}.npz")


@pytest.fixture
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    return torch.device("cuda", 0)
