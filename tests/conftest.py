from __future__ import annotations

import importlib
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

REPO = Path(__file__).resolve().parents[1]
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))

GOLDEN = Path(__file__).resolve().parent / "golden"
PACKAGE_NAME = "lumen-sosp26-ae_b200"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


def load_package():
    return importlib.import_module(PACKAGE_NAME)


@pytest.fixture(scope="session")
def pkg():
    """The product package with liblumen_b200.so built and loaded."""
    import __graft_entry__ as entry

    entry.build()
    return load_package()


@pytest.fixture(scope="session")
def cuda_pkg(pkg):
    if not torch.cuda.is_available():
        pytest.fail("a test marked gpu ran without a CUDA device")
    torch.cuda.set_device(0)
    pkg.clear_status()
    return pkg


def bf16_from_bits(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16)


def load_golden(name: str) -> dict:
    data = np.load(GOLDEN / f"{name}.npz")
    out = {}
    for key in data.files:
        arr = data[key]
        out[key] = bf16_from_bits(arr) if arr.dtype == np.uint16 else torch.from_numpy(arr.copy())
    return out


# tolerance of the operator outputs against the fp32-accumulated oracle
RTOL = 2e-2
ATOL = 2e-2
