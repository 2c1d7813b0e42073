import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a); parity tests through the C ABI")


@pytest.fixture(scope="session")
def oracle():
    from oracle import affine
    affine.lib()          # builds oracle/libg4q_oracle.so with make if it is missing
    return affine


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test collected without a CUDA device")
    from helios_b200 import _lib
    _lib.load()           # fails loudly when libg4q.so is missing: no fallback path exists
    torch.manual_seed(0)
    return torch.device("cuda", 0)


GOLDEN = ROOT / "tests" / "golden"
