import os
from pathlib import Path
import sys

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")


@pytest.fixture(scope="session")
def lib():
    """The in-tree native library; fails (never skips) when it is missing."""
    import paralyn_b200 as p
    return p.library()


@pytest.fixture(scope="session")
def reference_checkout():
    """The reference checkout (PARALYN_REFERENCE, else the oracle recipe's default);
    skips where there is none (GPU machines have no checkout)."""
    import oracle
    checkout = oracle.reference_checkout()
    if checkout is None:
        pytest.skip("reference checkout not present on this machine")
    return checkout


@pytest.fixture()
def context():
    import paralyn_b200 as p
    with p.Context("cuda:0") as ctx:
        yield ctx
