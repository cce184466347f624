import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and libkernels.so")


def golden(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz") as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def cuda():
    """The CUDA device for -m gpu tests; fails (never skips) without one."""
    import torch
    assert torch.cuda.is_available(), "gpu tests need a CUDA device"
    torch.cuda.init()
    return torch.device("cuda", 0)
