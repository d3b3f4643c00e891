from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 and the built sm_100a library")


@pytest.fixture(scope="session")
def cuda_lib():
    """Load the CUDA library for GPU tests; fail loudly if it is missing."""
    import torch

    from pagegauge_b200 import _lib

    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but CUDA is not available")
    return _lib.load()
