"""The TensorRT plugin's enqueue, relinked against liblocalcorr_b200.so.

tests/relink/plugin_enqueue_relink.cpp repeats the reference plugin's call of
launchLocalCorrCudaPyramidForward
(cuda_pyramid/localcorr_cuda_pyramid_plugin.cpp:164-199) against
include/localcorr_b200.h; here it is compiled with g++ and linked against the
built library, and its validation paths run without a GPU (an empty batch
succeeds, an invalid level count fails, a 3-D input fails) — none of them
reaches a CUDA call. The GPU test in test_gpu_parity.py runs a real enqueue.
"""

import ctypes
import shutil
import sys
from pathlib import Path

import pytest

sys.path.insert(0, str(Path(__file__).resolve().parent / "relink"))

from localcorr_b200 import _lib  # noqa: E402

ARGS = [ctypes.c_void_p] * 4 + [ctypes.c_int] * 9 + [ctypes.c_void_p]


def load_relink(tmp_dir):
    import build_relink

    so = build_relink.build(tmp_dir)
    lib = ctypes.CDLL(str(so))
    lib.relink_enqueue.restype = ctypes.c_int
    lib.relink_enqueue.argtypes = ARGS
    return lib


@pytest.fixture(scope="module")
def relink(tmp_path_factory):
    if shutil.which("g++") is None:
        pytest.skip("g++ not available")
    if not _lib.LIB_PATH.exists():
        pytest.skip("liblocalcorr_b200.so not built")
    return load_relink(tmp_path_factory.mktemp("relink"))


def test_plugin_enqueue_compiles_links_and_validates(relink):
    # empty batch: success without touching the device
    assert relink.relink_enqueue(None, None, None, None, 0, 8, 8, 64, 1, 4, 4, 1, 0, None) == 0
    # levels outside [1, 8]: the launcher's false becomes the plugin's 1
    assert relink.relink_enqueue(None, None, None, None, 1, 8, 8, 64, 1, 4, 0, 1, 0, None) == 1
    assert "levels" in _lib.last_error()
    # dilation < 1
    assert relink.relink_enqueue(None, None, None, None, 1, 8, 8, 64, 0, 4, 1, 0, 0, None) == 1
    assert "dilation" in _lib.last_error()
