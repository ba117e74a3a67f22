import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (sm_100a) and the built native library")


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    with np.load(ROOT / "tests" / "golden" / "templates.npz") as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a visible CUDA device")
    from devproc_b200 import _native
    _native.device_init(0)
    return torch.device("cuda", 0)
