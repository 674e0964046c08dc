"""Shared test setup: import paths, the `gpu` marker and golden-vector loading."""
import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "specdec-quant-triton_b200")
GOLDEN = os.path.join(REPO, "tests", "golden")
for p in (REPO, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU and the built libspecq.so")


def load_golden(name: str) -> dict:
    with np.load(os.path.join(GOLDEN, name + ".npz")) as z:
        return {k: z[k] for k in z.files}


@pytest.fixture
def golden():
    return load_golden


@pytest.fixture(scope="session")
def cuda():
    """Skip-free guard for GPU tests: fail loudly if the GPU or the library is missing."""
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import specq  # noqa: F401  (raises if libspecq.so is missing)
    major, _ = torch.cuda.get_device_capability()
    assert major == 10, "these kernels are built for sm_100a only"
    return torch.device("cuda:0")
