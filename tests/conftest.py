import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
for p in (ROOT / "oracle", ROOT / "vibevoice.cpp_b200", ROOT / "tests"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built libvvq2.so")


@pytest.fixture(scope="session")
def vv():
    """The product binding, on a machine with an sm_100 device (gpu tests)."""
    import vvq2
    assert vvq2.lib().vvq2_device_count() > 0, "no sm_100 device visible"
    return vvq2


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    def load(name):
        return np.load(GOLDEN / name)
    return load
