"""pytest configuration: the ``gpu`` marker and import paths.

CPU-only tests (``-m "not gpu"``) cover the oracle against the reference's
golden fixtures, the host-side logic of the package and the C ABI symbol
table. Tests marked ``gpu`` need a CUDA device and the built library and
check the CUDA engine against the oracle.
"""

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device and the built library")


@pytest.fixture(autouse=True)
def _restore_backend():
    import localcorr_b200.backend as backend

    saved = backend._onnx_backend
    yield
    backend._onnx_backend = saved
