"""Generate the golden fixtures of tests/golden/ from the reference itself.

Runs the reference package's own pure-PyTorch implementations (its
independent test references, tests/_reference.py:43-125, and its
standard-ops formulation, onnx_generic.py:58-198) on small seeded inputs
and stores inputs, outputs and autograd gradients as .npz files. The
fixtures pin the CPU oracle (tests/test_oracle_golden.py) and the CUDA
engine (tests/test_gpu_parity.py) to the reference's results.

Usage:
    python tests/golden/make_golden.py --reference <localcorr checkout dir>

The checkout directory is the reference package itself (its
pyproject maps the package name to the repository root), so it is made
importable as ``localcorr`` through a symlink in a temporary directory.
"""

from __future__ import annotations

import argparse
import math
import os
import sys
import tempfile
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent


def _import_reference(ref: Path):
    tmp = Path(tempfile.mkdtemp(prefix="lcref_"))
    (tmp / "localcorr").symlink_to(ref.resolve(), target_is_directory=True)
    sys.path.insert(0, str(tmp))
    sys.path.insert(0, str(ref.resolve() / "tests"))
    import localcorr.onnx_generic as onnx_generic  # noqa: E402
    import _reference  # noqa: E402

    return onnx_generic, _reference


def _np(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().numpy().astype(np.float32)


def pyramid_case(name, ref, gen, batch, channels, height, width, levels, radius, max_disp,
                 seed, far_oob=False):
    onnx_generic, R = ref
    f1, f2 = R.make_fmaps(batch=batch, channels=channels, height=height, width=width, seed=seed)
    coords = R.make_coords(batch=batch, height=height, width=width, max_disp=max_disp,
                           seed=seed + 1)
    if far_oob:
        # Rows whose windows fall completely outside every level, and columns
        # straddling the borders.
        coords[:, 0, 0, :] = 1000.0
        coords[:, 1, 1, :] = -500.0
        coords[:, 0, :, 0] = -6.5
        coords[:, 0, :, -1] = width + 3.25
    g = torch.Generator().manual_seed(seed + 2)
    f1r = f1.clone().requires_grad_(True)
    f2r = f2.clone().requires_grad_(True)
    out = R.pyramid_localcorr_reference(f1r, f2r, coords, levels, radius)
    block_out = out.reshape(batch, -1, height, width) / math.sqrt(channels)
    grad_out = torch.randn(block_out.shape, generator=g)
    g1, g2 = torch.autograd.grad(block_out, [f1r, f2r], grad_out)
    generic = onnx_generic.localcorr_pyramid_onnx_generic(f1, f2, coords, levels, radius)
    np.savez_compressed(
        OUT / f"{name}.npz",
        fmap1=_np(f1), fmap2=_np(f2), coords=_np(coords), grad_out=_np(grad_out),
        out_ref=_np(out), out_generic=_np(generic), grad_fmap1=_np(g1), grad_fmap2=_np(g2),
        levels=levels, radius=radius,
    )


def dilation_case(name, ref, batch, channels, height, width, radius, dilation, seed):
    _, R = ref
    f1, f2 = R.make_fmaps(batch=batch, channels=channels, height=height, width=width, seed=seed)
    out = R.shifted_spatial_reference(f1, f2, radius=radius, dilation=dilation, normalize=None)
    np.savez_compressed(OUT / f"{name}.npz", fmap1=_np(f1), fmap2=_np(f2), out_ref=_np(out),
                        radius=radius, dilation=dilation)


def spatial_case(name, ref, batch, channels, height, width, radius, seed):
    onnx_generic, R = ref
    i1, i2 = R.make_fmaps(batch=batch, channels=channels, height=height, width=width, seed=seed)
    a = i1.clone().requires_grad_(True)
    b = i2.clone().requires_grad_(True)
    out = R.spatial_corr_reference(a, b, radius)
    g = torch.Generator().manual_seed(seed + 2)
    grad_out = torch.randn(out.shape, generator=g)
    g1, g2 = torch.autograd.grad(out, [a, b], grad_out)
    generic = onnx_generic.spatial_corr_onnx_generic(i1, i2, radius)
    np.savez_compressed(OUT / f"{name}.npz", in1=_np(i1), in2=_np(i2), grad_out=_np(grad_out),
                        out_ref=_np(out), out_generic=_np(generic), grad_in1=_np(g1),
                        grad_in2=_np(g2), radius=radius)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reference", required=True, type=Path,
                    help="reference localcorr checkout (the package directory)")
    a = ap.parse_args(argv)
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    ref = _import_reference(a.reference)
    # Shapes of the reference's own CPU tests (tests/test_blocks.py:30-31,
    # tests/test_onnx_generic.py:22-23) plus an odd-sized 4-level r=4 case
    # with out-of-bounds windows, and a one-level r=1 case.
    pyramid_case("pyr_b2c8_16x24_l3r2", ref, None, 2, 8, 16, 24, 3, 2, 3.0, seed=20)
    pyramid_case("pyr_b1c16_17x21_l4r4_oob", ref, None, 1, 16, 17, 21, 4, 4, 8.0, seed=40,
                 far_oob=True)
    pyramid_case("pyr_b1c4_8x8_l1r1", ref, None, 1, 4, 8, 8, 1, 1, 1.5, seed=7)
    dilation_case("dil_b1c6_12x14_r3d2", ref, 1, 6, 12, 14, 3, 2, seed=23)
    spatial_case("spatial_b2c8_12x16_r4", ref, 2, 8, 12, 16, 4, seed=51)
    spatial_case("spatial_b1c3_10x12_r3", ref, 1, 3, 10, 12, 3, seed=3)
    for p in sorted(OUT.glob("*.npz")):
        print(p.name, p.stat().st_size)
    return 0


if __name__ == "__main__":
    sys.exit(main())
