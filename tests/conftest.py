import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU; run with -m gpu")


@pytest.fixture(scope="session")
def pkb():
    """The product's Python bindings, with the in-tree library loaded."""
    import libpktito_b200 as P
    P.lib()
    return P


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O
    O.olib()
    return O


@pytest.fixture(scope="session")
def cuda_device(pkb):
    """Fails (not skips) a GPU test when no sm_100 device is usable: the
    product has no CPU path to fall back to."""
    n = pkb.device_count()
    assert n > 0, "no sm_100 device visible to libpktito_b200"
    return 0
