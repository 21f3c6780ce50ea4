"""Build liblocalcorr_b200.so in-tree with nvcc for sm_100a.

Each .cu under this directory is compiled to an object file in
``localcorr_b200/_build/`` (in parallel), then linked into
``localcorr_b200/liblocalcorr_b200.so``. Objects are rebuilt only when a
source or header is newer than them.

``--bounds-check`` builds the same sources with ``-DLC_BOUNDS_CHECK`` into
``localcorr_b200/_build_checked/`` and ``liblocalcorr_b200_checked.so``
(device-side index checks; selected at import time by
``LOCALCORR_B200_BOUNDS_CHECK=1``).

Usage: python -m localcorr_b200.csrc.build [--force] [--verbose] [--bounds-check]
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

CSRC = Path(__file__).resolve().parent
PKG = CSRC.parent
ROOT = PKG.parent
INCLUDE = ROOT / "include"
BUILD = PKG / "_build"
LIB = PKG / "liblocalcorr_b200.so"
BUILD_CHECKED = PKG / "_build_checked"
LIB_CHECKED = PKG / "liblocalcorr_b200_checked.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-DLCB200_BUILD",
]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build")
    return cand


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _headers() -> list[Path]:
    return sorted(list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h")))


def _compile(src: Path, verbose: bool, extra: list[str], bdir: Path = BUILD) -> Path:
    obj = bdir / (src.stem + ".o")
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, *extra, f"-I{INCLUDE}", f"-I{CSRC}", "-c", str(src),
           "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout.strip() or res.stderr.strip()):
        print(res.stdout, res.stderr, flush=True)
    return obj


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False,
          bounds_check: bool = False) -> Path:
    """Build the library (``bounds_check``: the LC_BOUNDS_CHECK variant)."""
    bdir, lib = (BUILD_CHECKED, LIB_CHECKED) if bounds_check else (BUILD, LIB)
    bdir.mkdir(parents=True, exist_ok=True)
    srcs = _sources()
    newest_hdr = max((h.stat().st_mtime for h in _headers()), default=0.0)
    extra = ["-Xptxas", "-v"] if ptxas_verbose else []
    if bounds_check:
        extra = extra + ["-DLC_BOUNDS_CHECK"]
    todo = []
    for s in srcs:
        obj = bdir / (s.stem + ".o")
        if force or ptxas_verbose or not obj.exists() or obj.stat().st_mtime < max(
            s.stat().st_mtime, newest_hdr
        ):
            todo.append(s)
    if todo:
        workers = min(len(todo), max(1, os.cpu_count() or 1))
        with cf.ThreadPoolExecutor(workers) as ex:
            list(ex.map(lambda s: _compile(s, verbose or ptxas_verbose, extra, bdir), todo))
    objs = [bdir / (s.stem + ".o") for s in srcs]
    if force or todo or not lib.exists() or lib.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        tmp = lib.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs)]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, lib)
    return lib


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true",
                    help="print registers/spills/shared memory per kernel")
    ap.add_argument("--bounds-check", action="store_true",
                    help="build liblocalcorr_b200_checked.so (-DLC_BOUNDS_CHECK)")
    a = ap.parse_args(argv)
    path = build(force=a.force, verbose=a.verbose, ptxas_verbose=a.ptxas_verbose,
                 bounds_check=a.bounds_check)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
