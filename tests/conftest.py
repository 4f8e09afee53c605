import importlib
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

PKG_NAME = "gmdn-gated-muon-deltanet_b200"

# Every mixer-core call in the tests reads back the kernels' device status word
# (a bounded wait that gave up fails the test instead of passing silently).
os.environ.setdefault("GMDN_CHECK_STATUS", "1")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def load_pkg():
    """Import the product package (its directory name is not an identifier)."""
    return importlib.import_module(PKG_NAME)


@pytest.fixture(scope="session")
def pkg():
    return load_pkg()
