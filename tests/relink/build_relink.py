"""Compile tests/relink/plugin_enqueue_relink.cpp into a shared library linked
against liblocalcorr_b200.so (g++, the CUDA toolkit's headers only)."""

from __future__ import annotations

import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
PKG = ROOT / "localcorr_b200"
CUDA_INC = Path("/usr/local/cuda/include")


def build(out_dir: Path) -> Path:
    out = Path(out_dir) / "librelink_enqueue.so"
    cmd = ["g++", "-std=c++17", "-O1", "-fPIC", "-shared", "-Wall", "-Werror",
           f"-I{ROOT / 'include'}", f"-I{HERE}", f"-I{CUDA_INC}",
           str(HERE / "plugin_enqueue_relink.cpp"), f"-L{PKG}", "-llocalcorr_b200",
           f"-Wl,-rpath,{PKG}", "-o", str(out)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"relink build failed:\n{' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
    return out
