"""pytest configuration: the `gpu` marker and shared fixtures.

`-m "not gpu"` runs the oracle, host-logic and ABI-surface tests on any
machine; `-m gpu` runs the parity tests through libdct_cuda.so's C-ABI on a
B200.  GPU tests never fall back to the CPU: if the library or the device is
missing they fail.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

# the reference checkout: DCT_REFERENCE_DIR, else a `reference` directory beside
# this repository; the tests that need it skip when neither holds nn_engine.py
REFERENCE_DIR = os.environ.get("DCT_REFERENCE_DIR") or os.path.join(os.path.dirname(ROOT), "reference")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device and libdct_cuda.so (run on a B200)")
    config.addinivalue_line("markers", "reference: needs the reference sources (skipped when absent)")


@pytest.fixture(scope="session")
def reference_dir():
    if not os.path.isfile(os.path.join(REFERENCE_DIR, "nn_engine.py")):
        pytest.skip("reference sources not mounted")
    return REFERENCE_DIR


@pytest.fixture(scope="session")
def dev():
    """Device helper over libdct_cuda.so (GPU tests only)."""
    from tests.devhelp import Dev
    return Dev()
