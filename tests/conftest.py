"""Shared fixtures.  Tests marked ``gpu`` need an sm_100 device and call the kernels through
the C ABI; everything else runs on the CPU (oracle vs golden vectors, host logic, the
library's exports and host-side argument checks, gloo multi-rank logic)."""
from __future__ import annotations

import importlib
import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))

GOLDEN = REPO / "tests" / "golden" / "golden.npz"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU; runs the CUDA kernels")
    config.addinivalue_line("markers", "slow: longer CPU test")


@pytest.fixture(scope="session")
def pkg():
    return importlib.import_module("4d_ttt_merging_b200")


@pytest.fixture(scope="session")
def golden():
    with np.load(GOLDEN) as data:
        return {k: data[k] for k in data.files}


@pytest.fixture(scope="session")
def oracle():
    return importlib.import_module("oracle")


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("this test needs a CUDA device (run with -m 'not gpu' on a CPU-only machine)")
    major, minor = torch.cuda.get_device_capability(0)
    if major != 10:
        pytest.fail(f"this test needs an sm_100 device, found sm_{major}{minor}")
    return torch.device("cuda", 0)
