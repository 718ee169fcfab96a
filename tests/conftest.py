import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and the built CUDA library")


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    return np.load(ROOT / "tests" / "golden" / "qconv_kat.npz")


@pytest.fixture(scope="session")
def cuda_lib():
    """The CUDA library must load on a GPU box: no fallback, no skip."""
    import torch

    assert torch.cuda.is_available(), "GPU test run without a visible CUDA device"
    from my_own_cnn_b200 import _lib

    return _lib.lib()
