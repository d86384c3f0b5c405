import os
from pathlib import Path
import sys

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))
REFERENCE = Path("/root/reference")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")


@pytest.fixture(scope="session")
def lib():
    """The in-tree native library; fails (never skips) when it is missing."""
    import paralyn_b200 as p
    return p.library()


@pytest.fixture(scope="session")
def reference_checkout():
    if not (REFERENCE / "include" / "paralyn" / "native.h").exists():
        pytest.skip("reference checkout not present on this machine")
    return REFERENCE


@pytest.fixture()
def context():
    import paralyn_b200 as p
    with p.Context("cuda:0") as ctx:
        yield ctx
