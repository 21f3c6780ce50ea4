"""ctypes binding of liblocalcorr_b200.so (the C ABI in include/localcorr_b200.h).

The library is loaded once, from the package directory, where
``python -m localcorr_b200.csrc.build`` (or ``__graft_entry__.build()``) puts
it. There is no fallback: when the library is missing every CUDA op raises
ImportError, as the reference does for its unbuilt CUDA library
(blocks.py:552-565). With ``LOCALCORR_B200_BOUNDS_CHECK=1`` in the
environment the bounds-checked build (liblocalcorr_b200_checked.so, built
with ``--bounds-check``) is loaded instead.
"""

from __future__ import annotations

import ctypes
import logging
import os
from pathlib import Path

logger = logging.getLogger(__name__)

LIB_PATH_DEFAULT = Path(__file__).resolve().parent / "liblocalcorr_b200.so"
LIB_PATH_CHECKED = Path(__file__).resolve().parent / "liblocalcorr_b200_checked.so"
BOUNDS_CHECK = os.environ.get("LOCALCORR_B200_BOUNDS_CHECK", "") not in ("", "0")
LIB_PATH = LIB_PATH_CHECKED if BOUNDS_CHECK else LIB_PATH_DEFAULT

F32 = 0
F16 = 1
ACC_FMAP2 = 1  # backward: add into the float32 fmap2 gradient
ACC_FMAP1 = 2  # backward: add into the fmap1 gradient
ENGINE_AUTO = 0
ENGINE_SIMT = 1
ENGINE_TC = 2

_c_void_p = ctypes.c_void_p
_c_int = ctypes.c_int
_c_bool = ctypes.c_bool
_c_float = ctypes.c_float
_c_size_t = ctypes.c_size_t

# name -> (restype, argtypes). Every exported symbol of include/localcorr_b200.h.
PROTOTYPES = {
    "launchLocalCorrCudaPyramidForward": (
        _c_bool,
        [_c_void_p] * 4 + [_c_int] * 7 + [_c_bool, _c_bool, _c_void_p],
    ),
    "launchLocalCorrCudaPyramidBackward": (
        _c_bool,
        [_c_void_p] * 6 + [_c_int] * 7 + [_c_bool, _c_bool, _c_void_p],
    ),
    "localCorrB200PyramidWorkspaceBytes": (_c_size_t, [_c_int] * 9),
    "launchLocalCorrB200PyramidForward": (
        _c_bool,
        [_c_void_p] * 4
        + [_c_int] * 7
        + [_c_int, _c_int, _c_bool, _c_float, _c_int, _c_void_p, _c_size_t, _c_void_p],
    ),
    "launchLocalCorrB200PyramidBackward": (
        _c_bool,
        [_c_void_p] * 6
        + [_c_int] * 7
        + [_c_int, _c_int, _c_bool, _c_float, _c_int, _c_int, _c_void_p, _c_size_t, _c_void_p],
    ),
    "localCorrB200PyramidWorkspaceBytesMapDims": (_c_size_t, [_c_int] * 11),
    "launchLocalCorrB200PyramidForwardMapDims": (
        _c_bool,
        [_c_void_p] * 4
        + [_c_int] * 9
        + [_c_int, _c_int, _c_bool, _c_float, _c_int, _c_void_p, _c_size_t, _c_void_p],
    ),
    "launchLocalCorrB200PyramidBackwardMapDims": (
        _c_bool,
        [_c_void_p] * 6
        + [_c_int] * 9
        + [_c_int, _c_int, _c_bool, _c_float, _c_int, _c_int, _c_void_p, _c_size_t, _c_void_p],
    ),
    "localCorrB200PyramidSortStateBytes": (_c_size_t, [_c_int] * 11),
    "launchLocalCorrB200PyramidForwardKeepSort": (
        _c_bool,
        [_c_void_p] * 4
        + [_c_int] * 9
        + [_c_int, _c_int, _c_bool, _c_float, _c_int, _c_void_p, _c_size_t, _c_void_p,
           _c_size_t, _c_void_p],
    ),
    "launchLocalCorrB200PyramidBackwardWithSort": (
        _c_bool,
        [_c_void_p] * 6
        + [_c_int] * 9
        + [_c_int, _c_int, _c_bool, _c_float, _c_int, _c_int, _c_void_p, _c_size_t, _c_void_p,
           _c_size_t, _c_void_p],
    ),
    "launchLocalCorrB200PyramidForwardNoAlloc": (
        _c_bool,
        [_c_void_p] * 4 + [_c_int] * 6 + [_c_int, _c_int, _c_bool, _c_float, _c_void_p],
    ),
    "launchLocalCorrB200PyramidBuild": (
        _c_bool,
        [_c_void_p, _c_void_p] + [_c_int] * 6 + [_c_void_p],
    ),
    "launchLocalCorrB200PyramidBuildBackward": (
        _c_bool,
        [_c_void_p, _c_bool, _c_void_p] + [_c_int] * 6 + [_c_void_p],
    ),
    "launchLocalCorrB200NchwToNhwc": (_c_bool, [_c_void_p, _c_void_p] + [_c_int] * 4 + [_c_void_p]),
    "launchLocalCorrB200NhwcToNchw": (_c_bool, [_c_void_p, _c_void_p] + [_c_int] * 4 + [_c_void_p]),
    "launchLocalCorrB200SpatialForward": (
        _c_bool,
        [_c_void_p] * 3 + [_c_int] * 7 + [_c_float, _c_void_p],
    ),
    "launchLocalCorrB200SpatialBackward": (
        _c_bool,
        [_c_void_p] * 5 + [_c_int] * 7 + [_c_float, _c_void_p],
    ),
    "localCorrB200PyramidRecordsBytes": (_c_size_t, [_c_int] * 8),
    "launchLocalCorrB200PyramidBackwardFmap1": (
        _c_bool,
        [_c_void_p] * 5 + [_c_int] * 9 + [_c_bool, _c_float, _c_int, _c_void_p, _c_size_t,
                                          _c_void_p, _c_size_t, _c_void_p, _c_size_t, _c_void_p],
    ),
    "launchLocalCorrB200PyramidBackwardFmap2Pull": (
        _c_bool,
        [ctypes.POINTER(_c_void_p)] * 2 + [_c_int, _c_void_p] + [_c_int] * 8
        + [_c_float, _c_int, _c_void_p, _c_size_t, _c_void_p],
    ),
    "localCorrB200GetLastError": (ctypes.c_char_p, []),
    "localCorrB200DeviceStatus": (_c_int, [_c_int]),
    "localCorrB200Version": (_c_int, []),
    "localCorrB200LaunchCount": (ctypes.c_longlong, [_c_int]),
    "localCorrB200SetDeterministic": (None, [_c_int]),
    "localCorrB200GetDeterministic": (_c_int, []),
    "localCorrB200BoundsViolations": (ctypes.c_longlong, [_c_int]),
}

_LIB = None
_LIB_LOADED = False


def load_library(path: Path | str | None = None):
    """Load (once) and return the ctypes handle of liblocalcorr_b200.so, or None.

    Returns None when the file does not exist or cannot be loaded; the
    loading error is logged. Every prototype in PROTOTYPES is bound; a
    missing symbol makes the library unusable (returns None).
    """
    global _LIB, _LIB_LOADED
    if path is None and _LIB_LOADED:
        return _LIB
    p = Path(path) if path is not None else LIB_PATH
    lib = None
    if p.exists():
        try:
            lib = ctypes.CDLL(str(p))
            for name, (res, args) in PROTOTYPES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
        except (OSError, AttributeError) as exc:
            logger.warning("could not load %s (%s)", p, exc)
            lib = None
    if path is None:
        _LIB, _LIB_LOADED = lib, True
    return lib


def require_library():
    """Return the loaded library or raise ImportError with the build command."""
    lib = load_library()
    if lib is None:
        raise ImportError(
            "the localcorr_b200 CUDA library (liblocalcorr_b200.so) has not been built "
            "(or could not be loaded). Build it with: python -m localcorr_b200.csrc.build"
        )
    return lib


def last_error(lib=None) -> str:
    lib = lib or load_library()
    if lib is None:
        return "library not loaded"
    msg = lib.localCorrB200GetLastError()
    return msg.decode() if msg else ""


def check(ok: bool, what: str, lib=None) -> None:
    """Raise RuntimeError with the library's message when a launcher failed."""
    if not ok:
        raise RuntimeError(f"localcorr_b200 {what} failed: {last_error(lib)}")
