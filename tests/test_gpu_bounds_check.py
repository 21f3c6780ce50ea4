"""The bounds-checked build (LC_BOUNDS_CHECK) over the edge cases.

``compute-sanitizer`` is closed on this pool; in its place the library is
also built with every data-dependent global index checked on the device
(liblocalcorr_b200_checked.so, ``build --bounds-check``). These tests run
that build over small exhaustive cases (odd sizes, levels down to 1-pixel
maps, r in {0, 1, 3, 4, 8}, dilation, far out-of-bounds and converging
coords, both engines, the spatial kernels) and require (a) no recorded
violation and (b) the same results as the normal build (float tolerance:
the checks skip nothing when no index is out of range, so only the order of
atomic adds may differ). A planted bug is never run on the GPU: the failure
path (violation -> false -> RuntimeError naming the site) is the same
host code as any failed launch.
"""

import pytest
import torch

from localcorr_b200 import _lib, ops
from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def libs():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    normal = _lib.load_library()
    assert normal is not None
    if not _lib.LIB_PATH_CHECKED.exists():
        pytest.skip("bounds-checked library not built (build --bounds-check)")
    checked = _lib.load_library(_lib.LIB_PATH_CHECKED)
    assert checked is not None and checked.localCorrB200BoundsViolations(1) == 0
    return normal, checked


def _run_both(libs, fn):
    """fn() with the normal library, then with the checked one."""
    normal, checked = libs
    saved = _lib._LIB
    out_n = fn()
    try:
        _lib._LIB = checked
        out_c = fn()
        torch.cuda.synchronize()
    finally:
        _lib._LIB = saved
    assert checked.localCorrB200BoundsViolations(1) == 0
    assert normal.localCorrB200BoundsViolations(0) == -1
    return out_n, out_c


def _coords(kind, b, h, w, seed):
    if kind == "oob":
        return oracle.make_coords_gauss_oob(b, h, w, 6.0, 0.3, seed=seed)
    if kind == "far":
        c = oracle.make_coords_uniform(b, h, w, 4.0, seed=seed)
        c[:, :, ::3] += 1e4  # whole rows of pixels far outside the map
        c[:, :, 1::5] -= 3e3
        return c
    if kind == "converge":
        g = torch.Generator().manual_seed(seed)
        c = torch.empty(b, 2, h, w)
        c[:, 0] = w / 2 + torch.rand(b, h, w, generator=g) * 2
        c[:, 1] = h / 2 + torch.rand(b, h, w, generator=g) * 2
        return c
    return oracle.make_coords_uniform(b, h, w, 6.0, seed=seed)


PYR_CASES = [
    # b, c, h, w, levels, radius, dilation, dtype, coords kind
    (2, 128, 33, 47, 4, 4, 1, torch.float16, "oob"),      # tensor-core engine
    (1, 256, 24, 40, 3, 3, 1, torch.float16, "converge"),
    (1, 64, 19, 29, 2, 8, 1, torch.float16, "far"),
    (1, 64, 32, 32, 1, 4, 1, torch.float16, "uniform"),
    (2, 24, 17, 23, 5, 4, 1, torch.float32, "oob"),       # CUDA-core engine
    (1, 7, 9, 13, 4, 0, 1, torch.float32, "uniform"),
    (1, 16, 8, 8, 4, 1, 1, torch.float32, "far"),         # level 3 is 1x1
    (1, 12, 15, 21, 3, 3, 2, torch.float16, "oob"),       # dilation 2
    (1, 33, 16, 16, 5, 8, 1, torch.float16, "converge"),  # odd C: CUDA-core
]


@pytest.mark.parametrize("case", PYR_CASES,
                         ids=lambda c: "b{}c{}_{}x{}_l{}r{}d{}_{}_{}".format(
                             *c[:7], str(c[7]).split(".")[-1], c[8]))
def test_pyramid_checked_build_matches(libs, case):
    b, c, h, w, levels, r, dil, dtype, kind = case
    f1, f2 = oracle.make_fmaps(b, c, h, w, seed=3)
    co = _coords(kind, b, h, w, seed=4).to(DEV, dtype)
    fm1 = ops.nchw_to_nhwc(f1.to(DEV, dtype))
    packed = ops.pyramid_build(f2.to(DEV, dtype), levels)
    rd = 2 * r + 1
    gout = torch.randn(b, levels, rd * rd, h, w,
                       generator=torch.Generator().manual_seed(5)).to(DEV, dtype)

    def run():
        out = ops.pyramid_corr_forward(fm1, packed, co, r, levels, dil, False, 0.5)
        g1, g2 = ops.pyramid_corr_backward(fm1, packed, co, gout, r, levels, dil, False, 0.5)
        return out.float(), g1.float(), g2

    n, k = _run_both(libs, run)
    tol = dict(rtol=1e-5, atol=1e-5) if dtype == torch.float32 else dict(rtol=1e-3, atol=1e-3)
    for x, y in zip(n, k):
        torch.testing.assert_close(y, x, **tol)


@pytest.mark.parametrize("case", [(2, 16, 12, 20, 3, 1, torch.float32),
                                  (1, 24, 9, 13, 4, 2, torch.float16),
                                  (1, 8, 16, 32, 2, 3, torch.float32),
                                  (2, 12, 10, 14, 1, 1, torch.float16)],
                         ids=lambda c: "b{}c{}_{}x{}_r{}d{}_{}".format(
                             *c[:6], str(c[6]).split(".")[-1]))
def test_spatial_checked_build_matches(libs, case):
    b, c, h, w, r, dil, dtype = case
    f1, f2 = oracle.make_fmaps(b, c, h, w, seed=7)
    a, bb = f1.to(DEV, dtype), f2.to(DEV, dtype)
    rd = 2 * r + 1
    g = torch.randn(b, rd, rd, h, w, generator=torch.Generator().manual_seed(8)).to(DEV, dtype)

    def run():
        out = ops.spatial_forward(a, bb, r, dil, 0.25)
        g1, g2 = ops.spatial_backward(a, bb, g, r, dil, 0.25)
        return out.float(), g1.float(), g2.float()

    n, k = _run_both(libs, run)
    for x, y in zip(n, k):
        torch.testing.assert_close(y, x, rtol=0, atol=0)


def test_keep_sort_and_deterministic_paths_checked(libs):
    b, c, h, w, levels, r = 2, 128, 30, 44, 4, 4
    f1, f2 = oracle.make_fmaps(b, c, h, w, seed=9)
    co = _coords("oob", b, h, w, seed=10).to(DEV, torch.float16)
    fm1 = ops.nchw_to_nhwc(f1.to(DEV).half())
    packed = ops.pyramid_build(f2.to(DEV).half(), levels)
    gout = torch.randn(b, levels, 81, h, w, generator=torch.Generator().manual_seed(11)).to(
        DEV, torch.float16)
    normal, checked = libs

    def run():
        st = torch.empty(ops.sort_state_bytes(fm1, packed, r, levels), dtype=torch.uint8,
                         device=DEV)
        out = ops.pyramid_corr_forward(fm1, packed, co, r, levels, scale=0.5, sort_state=st)
        g1, g2 = ops.pyramid_corr_backward(fm1, packed, co, gout, r, levels, scale=0.5,
                                           sort_state=st)
        return out.float(), g1.float(), g2

    # the package pushes the mode into the library it holds; the checked one
    # is switched directly
    ops.set_deterministic(True)
    checked.localCorrB200SetDeterministic(1)
    try:
        n, k = _run_both(libs, run)
    finally:
        ops.set_deterministic(False)
        checked.localCorrB200SetDeterministic(0)
    for x, y in zip(n, k):
        assert torch.equal(x, y)


def test_deferred_fmap2_pull_checked(libs):
    # grad_fmap1 with kept records for 3 lookups, then one grad_fmap2 pull
    b, c, h, w, levels, r = 2, 128, 30, 44, 4, 4
    f1, f2 = oracle.make_fmaps(b, c, h, w, seed=12)
    fm1 = ops.nchw_to_nhwc(f1.to(DEV).half())
    packed = ops.pyramid_build(f2.to(DEV).half(), levels)
    cos = [_coords(kind, b, h, w, seed=13 + i).to(DEV, torch.float16)
           for i, kind in enumerate(("oob", "far", "converge"))]
    g = torch.Generator().manual_seed(14)
    gouts = [torch.randn(b, levels, 81, h, w, generator=g).to(DEV, torch.float16) for _ in cos]

    def run():
        g1 = torch.empty_like(fm1)
        g2 = torch.empty(packed.shape, dtype=torch.float32, device=DEV)
        states, recs = [], []
        for i, (co, go) in enumerate(zip(cos, gouts)):
            st = torch.empty(ops.sort_state_bytes(fm1, packed, r, levels), dtype=torch.uint8,
                             device=DEV)
            ops.pyramid_corr_forward(fm1, packed, co, r, levels, scale=0.5, sort_state=st)
            rec = torch.empty(ops.records_bytes(fm1, packed, r, levels), dtype=torch.uint8,
                              device=DEV)
            ops.pyramid_corr_backward_fmap1(fm1, packed, co, go, r, levels, 0.5, g1,
                                            _lib.ACC_FMAP1 if i else 0, st, rec)
            states.append(st)
            recs.append(rec)
        ops.pyramid_corr_backward_fmap2_pull(fm1, g2, r, levels, 0.5, states, recs, 0)
        return g1.float(), g2

    n, k = _run_both(libs, run)
    for x, y in zip(n, k):
        torch.testing.assert_close(y, x, rtol=1e-3, atol=1e-3)
