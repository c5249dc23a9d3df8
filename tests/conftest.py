import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "orbi-streammoe_b200")
for p in (ROOT, PKG, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests"),
          os.path.join(ROOT, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def port():
    import pyoracle

    if not os.path.exists(pyoracle.PORT_LIB):
        pyoracle.build()
    return pyoracle.Oracle("port")


@pytest.fixture(scope="session")
def ref():
    import pyoracle

    if not pyoracle.ref_available():
        pytest.skip("reference compiled in place (oracle/_ref) not available")
    return pyoracle.Oracle("reference")


@pytest.fixture(scope="session")
def golden_dir():
    return os.path.join(ROOT, "tests", "golden")
