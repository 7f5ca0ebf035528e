import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

# the reference checkout: $SEPIA_REFERENCE, else a "reference" directory beside the repository
REFERENCE = Path(os.environ.get("SEPIA_REFERENCE", str(ROOT.parent / "reference")))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (runs the sm_100a kernels)")


def cuda_ok() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def lib():
    """The CUDA library; on a GPU box a missing library is a failure, not a skip."""
    if not cuda_ok():
        pytest.skip("no CUDA device")
    from sepia_b200 import lib as L
    return L.load()


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O
    O.build()
    return O


@pytest.fixture(scope="session")
def reference_dir():
    if not (REFERENCE / "src" / "sepia.c").exists():
        pytest.skip("reference checkout not present")
    return REFERENCE
