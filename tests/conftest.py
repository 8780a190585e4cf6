import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a); run with -m gpu")
    config.addinivalue_line("markers", "slow: full BASELINE-size case")


@pytest.fixture(scope="session")
def gpu():
    """A CudaGpu on device 0.  GPU tests fail loudly (no skip) when the device
    or the extension is missing: they only run under -m gpu on a B200."""
    from soso_b200.dispatch import CudaGpu
    g = CudaGpu(0)
    yield g
    g.close()
