"""C ABI checks that need no GPU: the library loads, exports every symbol
that include/localcorr_b200.h declares with the ctypes prototypes the
package binds, and rejects invalid configurations the way the reference
launchers do (cuda_pyramid/localcorr_cuda_pyramid_kernel.cu:1420-1435)
before any CUDA call."""

import ctypes
import re
from pathlib import Path

import pytest

from localcorr_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "localcorr_b200.h"


def _declared_symbols():
    text = HEADER.read_text()
    return re.findall(r"LCB200_API\s+[\w\s\*]+?\b(\w+)\s*\(", text)


@pytest.fixture(scope="module")
def lib():
    if not _lib.LIB_PATH.exists():
        from localcorr_b200.csrc import build

        build.build()
    handle = _lib.load_library()
    assert handle is not None, "liblocalcorr_b200.so failed to load"
    return handle


def test_header_declares_reference_launchers():
    syms = _declared_symbols()
    assert "launchLocalCorrCudaPyramidForward" in syms
    assert "launchLocalCorrCudaPyramidBackward" in syms
    assert len(syms) == len(set(syms))


def test_every_declared_symbol_is_exported_and_bound(lib):
    raw = ctypes.CDLL(str(_lib.LIB_PATH))
    for name in _declared_symbols():
        assert hasattr(raw, name), f"{name} not exported"
        assert name in _lib.PROTOTYPES, f"{name} has no ctypes prototype"
    assert set(_lib.PROTOTYPES) == set(_declared_symbols())


def test_reference_argtypes_match_reference_loader(lib):
    # blocks.py:100-121 of the reference binds these argtypes.
    fwd = _lib.PROTOTYPES["launchLocalCorrCudaPyramidForward"][1]
    bwd = _lib.PROTOTYPES["launchLocalCorrCudaPyramidBackward"][1]
    assert fwd == [ctypes.c_void_p] * 4 + [ctypes.c_int] * 7 + [ctypes.c_bool, ctypes.c_bool,
                                                                ctypes.c_void_p]
    assert bwd == [ctypes.c_void_p] * 6 + [ctypes.c_int] * 7 + [ctypes.c_bool, ctypes.c_bool,
                                                                ctypes.c_void_p]


def test_version_and_error_getters(lib):
    assert lib.localCorrB200Version() >= 100
    assert isinstance(_lib.last_error(lib), str)
    assert lib.localCorrB200LaunchCount(0) >= 0


def test_deterministic_mode_switch(lib):
    import torch

    import localcorr_b200 as lc

    assert lib.localCorrB200GetDeterministic() == 0
    lc.set_deterministic(True)
    try:
        assert lib.localCorrB200GetDeterministic() == 1 and lc.is_deterministic()
    finally:
        lc.set_deterministic(False)
    assert lib.localCorrB200GetDeterministic() == 0
    torch.use_deterministic_algorithms(True)
    try:
        assert lc.is_deterministic()
    finally:
        torch.use_deterministic_algorithms(False)
    assert not lc.is_deterministic()


def _fwd(lib, **kw):
    a = dict(B=1, H=16, W=16, C=8, r=2, L=3, dil=1, half=False, ymajor=False)
    a.update(kw)
    return lib.launchLocalCorrCudaPyramidForward(None, None, None, None, a["B"], a["H"], a["W"],
                                                 a["C"], a["r"], a["L"], a["dil"], a["half"],
                                                 a["ymajor"], None)


@pytest.mark.parametrize("kw", [dict(B=0), dict(H=0), dict(W=0), dict(B=-1)])
def test_empty_problem_is_a_successful_noop(lib, kw):
    assert _fwd(lib, **kw) is True


@pytest.mark.parametrize(
    "kw,msg",
    [
        (dict(L=0), "levels"),
        (dict(L=9), "levels"),
        (dict(dil=0), "dilation"),
        (dict(r=-1), "radius"),
        (dict(C=0), "C must be positive"),
        (dict(H=4, W=64, L=4), "empty"),
    ],
)
def test_invalid_configuration_returns_false_with_message(lib, kw, msg):
    assert _fwd(lib, **kw) is False
    assert msg in _lib.last_error(lib)


def test_backward_validation_matches_forward(lib):
    ok = lib.launchLocalCorrCudaPyramidBackward(None, None, None, None, None, None, 1, 16, 16, 8,
                                                2, 0, 1, False, False, None)
    assert ok is False and "levels" in _lib.last_error(lib)
    ok = lib.launchLocalCorrCudaPyramidBackward(None, None, None, None, None, None, 0, 16, 16, 8,
                                                2, 3, 1, False, False, None)
    assert ok is True


def test_extended_launcher_rejects_bad_dtype(lib):
    ok = lib.launchLocalCorrB200PyramidForward(None, None, None, None, 1, 8, 8, 4, 1, 1, 1, 7, 0,
                                               False, 1.0, 0, None, 0, None)
    assert ok is False and "dtype" in _lib.last_error(lib)
    ok = lib.launchLocalCorrB200PyramidForward(None, None, None, None, 1, 8, 8, 4, 1, 1, 1, 0, 5,
                                               False, 1.0, 0, None, 0, None)
    assert ok is False and "coords dtype" in _lib.last_error(lib)


def test_workspace_query_is_zero_for_invalid(lib):
    assert lib.localCorrB200PyramidWorkspaceBytes(1, 8, 8, 4, 1, 0, 1, 0, 0) == 0


def test_spatial_validation(lib):
    ok = lib.launchLocalCorrB200SpatialForward(None, None, None, 1, 4, 8, 8, -1, 1, 0, 1.0, None)
    assert ok is False
    ok = lib.launchLocalCorrB200SpatialForward(None, None, None, 0, 4, 8, 8, 4, 1, 0, 1.0, None)
    assert ok is True


def test_map_dims_launchers_validate_the_map_size(lib):
    # the map's levels must be non-empty: a 4-row map has no level 3
    ok = lib.launchLocalCorrB200PyramidForwardMapDims(None, None, None, None, 1, 16, 16, 4, 64,
                                                      8, 2, 4, 1, 0, 0, False, 1.0, 0, None, 0,
                                                      None)
    assert ok is False and "empty" in _lib.last_error(lib)
    ok = lib.launchLocalCorrB200PyramidBackwardMapDims(None, None, None, None, None, None, 1, 16,
                                                       16, 64, 4, 8, 2, 4, 1, 0, 0, False, 1.0, 0,
                                                       0, None, 0, None)
    assert ok is False and "empty" in _lib.last_error(lib)
    # an empty pixel band is a successful no-op whatever the map
    ok = lib.launchLocalCorrB200PyramidForwardMapDims(None, None, None, None, 1, 0, 16, 64, 64, 8,
                                                      2, 4, 1, 0, 0, False, 1.0, 0, None, 0,
                                                      None)
    assert ok is True
    assert lib.localCorrB200PyramidWorkspaceBytesMapDims(1, 16, 16, 4, 64, 8, 2, 4, 1, 0, 0) == 0


def test_map_dims_prototypes_extend_the_plain_ones():
    fwd = _lib.PROTOTYPES["launchLocalCorrB200PyramidForward"][1]
    fwd2 = _lib.PROTOTYPES["launchLocalCorrB200PyramidForwardMapDims"][1]
    assert fwd2[:7] == fwd[:7] and fwd2[7:9] == [ctypes.c_int] * 2 and fwd2[9:] == fwd[7:]
    bwd = _lib.PROTOTYPES["launchLocalCorrB200PyramidBackward"][1]
    bwd2 = _lib.PROTOTYPES["launchLocalCorrB200PyramidBackwardMapDims"][1]
    assert bwd2[:9] == bwd[:9] and bwd2[9:11] == [ctypes.c_int] * 2 and bwd2[11:] == bwd[9:]


def test_bounds_checked_build_loads_by_environment(tmp_path):
    """LOCALCORR_B200_BOUNDS_CHECK=1 selects liblocalcorr_b200_checked.so,
    which exports the same symbols and counts violations (the normal build
    reports -1)."""
    import os
    import subprocess
    import sys

    from localcorr_b200.csrc import build

    build.build(bounds_check=True)
    code = (
        "from localcorr_b200 import _lib\n"
        "lib = _lib.load_library()\n"
        "assert lib is not None\n"
        "print(_lib.LIB_PATH.name, lib.localCorrB200BoundsViolations(0))\n"
    )
    env = dict(os.environ, LOCALCORR_B200_BOUNDS_CHECK="1")
    res = subprocess.run([sys.executable, "-c", code], cwd=ROOT, env=env, capture_output=True,
                         text=True, timeout=300)
    assert res.returncode == 0, res.stderr
    assert res.stdout.split() == ["liblocalcorr_b200_checked.so", "0"]
    assert _lib.load_library().localCorrB200BoundsViolations(0) == -1
    raw = ctypes.CDLL(str(_lib.LIB_PATH_CHECKED))
    for name in _declared_symbols():
        assert hasattr(raw, name), f"{name} not exported by the checked build"


def test_deferred_fmap2_entry_points_validate_before_any_cuda_call(lib):
    import ctypes as ct

    # a pull over lookups needs their sort states and records
    ok = lib.launchLocalCorrB200PyramidBackwardFmap2Pull(
        None, None, 3, None, 1, 16, 16, 16, 16, 64, 4, 2, 0.125, 0, None, 0, None)
    assert ok is False
    assert "sort states and records" in _lib.last_error(lib)
    # empty problems are successful no-ops, as for the other launchers
    arr = (ct.c_void_p * 1)(None)
    assert lib.launchLocalCorrB200PyramidBackwardFmap2Pull(
        arr, arr, 0, None, 0, 16, 16, 16, 16, 64, 4, 2, 0.125, 0, None, 0, None) is True
    # the grad_fmap1 call takes float16 maps and coords of dtype 0 or 1 only
    ok = lib.launchLocalCorrB200PyramidBackwardFmap1(
        None, None, None, None, None, 1, 16, 16, 16, 16, 64, 4, 2, 7, False, 0.125, 0,
        None, 0, None, 0, None, 0, None)
    assert ok is False
    assert "coords dtype" in _lib.last_error(lib)
    # an invalid configuration has no records
    assert lib.localCorrB200PyramidRecordsBytes(1, 16, 16, 16, 16, 64, 4, 0) == 0
