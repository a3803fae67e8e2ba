import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU; runs through the C ABI")
    config.addinivalue_line("markers", "slow: full-size (BASELINE config) case")


@pytest.fixture(scope="session")
def ctx():
    """One device context per test session (GPU tests only)."""
    import zero_b200 as zb

    c = zb.Context(device=int(os.environ.get("ZGPU_DEVICE", "0")))
    yield c
    c.close()


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    return np.load(ROOT / "tests" / "golden" / "packer_golden.npz")
