import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU; run with -m gpu")


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    return dict(np.load(ROOT / "tests" / "golden" / "attention_golden.npz"))


@pytest.fixture(scope="session")
def ctfa():
    """The product library (raises if it is not built)."""
    from cudatransformer_b200 import _lib

    return _lib.load()


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    major, minor = torch.cuda.get_device_capability(0)
    assert (major, minor) == (10, 0), f"GPU tests need sm_100 (B200), found sm_{major}{minor}"
    return torch.device("cuda:0")
