"""Shared pytest setup.

Markers: `gpu` -- needs a CUDA device (run with `-m gpu` on a B200; the CPU
suite runs with `-m "not gpu"`).  GPU tests never skip silently when the
native library is missing: they fail, because the product path has no
CPU fallback.
"""
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the native library")


@pytest.fixture(scope="session")
def golden():
    def load(name):
        return dict(np.load(GOLDEN / name, allow_pickle=False))
    return load


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but CUDA is not available")
    from cign_b200 import _lib
    _lib.load_library()  # fails loudly if the native library is missing
    torch.backends.cuda.matmul.allow_tf32 = False
    return torch.device("cuda", 0)
