import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "nimformers-framework_b200")
for p in (PKG, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def nimf_gpu():
    """The CUDA library initialised on device 0 (GPU tests only)."""
    import nimf
    nimf.init(0)
    yield nimf


@pytest.fixture(scope="session")
def nimf_mod():
    """The host mirror with the library loaded but no device bound (host-only
    entry points such as the .nimq reader)."""
    import nimf
    nimf.lib()
    return nimf
