import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def _reference_root() -> Path:
    """The reference tree for the CPU pins: $DH_REFERENCE_ROOT, else the tree
    the oracle build compiled (oracle/_ref/REFERENCE_ROOT); a path that does
    not exist when neither is set, so the pins that need the tree skip."""
    env = os.environ.get("DH_REFERENCE_ROOT")
    if env:
        return Path(env)
    recorded = ROOT / "oracle" / "_ref" / "REFERENCE_ROOT"
    if recorded.is_file():
        return Path(recorded.read_text().strip())
    return ROOT / "oracle" / "_ref" / "no-reference-tree"


REFERENCE_ROOT = _reference_root()


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
