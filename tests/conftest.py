import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

REFERENCE_ROOT = Path(os.environ.get("DH_REFERENCE_ROOT", "/root/reference"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built libdh_b200.so")


@pytest.fixture(scope="session")
def cuda():
    """torch with a CUDA device; GPU tests fail loudly if the native library is missing."""
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from diffusionhard_b200 import _lib

    _lib.lib()  # raises DHLibraryError if libdh_b200.so is missing
    torch.cuda.init()
    return torch


def load_npz_cases(name):
    data = np.load(GOLDEN / name)
    cases = {}
    for key in data.files:
        case, field = key.split("__", 1)
        cases.setdefault(case, {})[field] = data[key]
    return cases


@pytest.fixture(scope="session")
def golden():
    return GOLDEN
