"""Tensor-core engine (tcgen05/TMA) parity: forward against the float64 oracle
and against the SIMT engine, across flow fields that stress the pixel sort
(i.i.d. Gaussian flow with far out-of-bounds pixels, smooth flow, uniform
+-64 flow, converging flow that overfills one anchor cell), radii, channel
counts, level counts, channel orders and coords dtypes. Float16 tolerance:
rtol 1e-2 / atol 1e-2 against the oracle on the same float16 inputs."""

import math

import pytest
import torch

from localcorr_b200 import _lib, ops
from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda"
F16TOL = dict(rtol=1e-2, atol=1e-2)


@pytest.fixture(scope="module", autouse=True)
def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    assert _lib.load_library() is not None


@pytest.fixture(autouse=True)
def _device_status_clean():
    lib = _lib.load_library()
    lib.localCorrB200DeviceStatus(1)
    yield
    assert lib.localCorrB200DeviceStatus(1) == 0, "a tensor-core pipeline wait timed out"


def _coords(kind, b, h, w, seed):
    if kind == "gauss_oob":
        return oracle.make_coords_gauss_oob(b, h, w, 6.0, 0.05, seed=seed)
    if kind == "smooth":
        return oracle.make_coords_smooth(b, h, w, 40.0, seed=seed)
    if kind == "uniform64":
        return oracle.make_coords_uniform(b, h, w, 64.0, seed=seed)
    if kind == "converge":
        # Every pixel looks at (almost) the same spot: one anchor cell gets
        # all of them (many 128-pixel chunks), the rest stay empty.
        g = torch.Generator().manual_seed(seed)
        c = torch.empty(b, 2, h, w)
        c[:, 0] = w / 2 + torch.rand(b, h, w, generator=g) * 3
        c[:, 1] = h / 2 + torch.rand(b, h, w, generator=g) * 3
        return c
    return oracle.make_coords_uniform(b, h, w, 8.0, seed=seed)


def _inputs(b, c, h, w, levels, kind, seed=0):
    f1, f2 = oracle.make_fmaps(b, c, h, w, seed=seed)
    f1, f2 = f1.half(), f2.half()
    co = _coords(kind, b, h, w, seed + 1)
    fm1 = ops.nchw_to_nhwc(f1.to(DEV))
    packed = ops.pyramid_build(f2.to(DEV), levels)
    return f1, f2, co, fm1, packed


CASES = [
    # b, c, h, w, levels, radius, coords
    (2, 256, 40, 52, 4, 4, "gauss_oob"),
    (1, 256, 47, 61, 4, 4, "smooth"),
    (2, 128, 32, 64, 4, 4, "uniform64"),
    (1, 128, 33, 70, 4, 3, "gauss_oob"),
    (1, 128, 30, 40, 4, 8, "uniform64"),
    (1, 64, 24, 36, 2, 4, "uniform8"),
    (1, 192, 20, 28, 1, 4, "uniform8"),
    (1, 256, 24, 40, 3, 3, "converge"),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "b{}c{}_{}x{}_l{}r{}_{}".format(*c))
def test_tc_forward_vs_oracle(case):
    b, c, h, w, levels, r, kind = case
    f1, f2, co, fm1, packed = _inputs(b, c, h, w, levels, kind)
    co16 = co.half()
    ref = oracle.pyramid_corr(f1.float(), f2.float(), co16.float(), levels, r)
    scale = 1.0 / math.sqrt(c)
    out = ops.pyramid_corr_forward(fm1, packed, co16.to(DEV), r, levels, 1, False, scale,
                                   _lib.ENGINE_TC)
    torch.testing.assert_close(out.double().cpu(), ref * scale, **F16TOL)
    simt = ops.pyramid_corr_forward(fm1, packed, co16.to(DEV), r, levels, 1, False, scale,
                                    _lib.ENGINE_SIMT)
    torch.testing.assert_close(out.float(), simt.float(), rtol=2e-3, atol=2e-3)


def test_tc_forward_ymajor_and_fp32_coords():
    b, c, h, w, levels, r = 1, 128, 36, 44, 3, 4
    f1, f2, co, fm1, packed = _inputs(b, c, h, w, levels, "gauss_oob", seed=3)
    ref = oracle.pyramid_corr(f1.float(), f2.float(), co, levels, r, ymajor=True)
    out = ops.pyramid_corr_forward(fm1, packed, co.to(DEV), r, levels, 1, True, 1.0,
                                   _lib.ENGINE_TC)
    torch.testing.assert_close(out.double().cpu() / math.sqrt(c), ref / math.sqrt(c), **F16TOL)


def test_tc_forward_all_out_of_bounds_is_zero():
    b, c, h, w, levels, r = 1, 64, 16, 32, 4, 4
    f1, f2, co, fm1, packed = _inputs(b, c, h, w, levels, "uniform8")
    co = torch.full((b, 2, h, w), 5000.0, dtype=torch.float16)
    out = ops.pyramid_corr_forward(fm1, packed, co.to(DEV), r, levels, 1, False, 1.0,
                                   _lib.ENGINE_TC)
    assert torch.count_nonzero(out) == 0


def test_tc_forward_repeatable():
    b, c, h, w, levels, r = 2, 256, 40, 52, 4, 4
    f1, f2, co, fm1, packed = _inputs(b, c, h, w, levels, "gauss_oob", seed=5)
    a = ops.pyramid_corr_forward(fm1, packed, co.half().to(DEV), r, levels, 1, False, 1.0,
                                 _lib.ENGINE_TC)
    bb = ops.pyramid_corr_forward(fm1, packed, co.half().to(DEV), r, levels, 1, False, 1.0,
                                  _lib.ENGINE_TC)
    assert torch.equal(a, bb)


def test_tc_reference_abi_uses_library_scratch():
    # The reference-compatible launcher takes no workspace: the library's
    # own stream-ordered scratch serves the tensor-core engine.
    import localcorr_b200 as lc

    b, c, h, w, levels, r = 1, 256, 30, 50, 4, 4
    f1, f2, co, fm1, packed = _inputs(b, c, h, w, levels, "gauss_oob", seed=6)
    out = lc.LocalCorrCudaPyramidFunction.apply(fm1, packed, co.half().to(DEV), r, levels, 1,
                                                False)
    ref = oracle.pyramid_corr(f1.float(), f2.float(), co.half().float(), levels, r)
    torch.testing.assert_close(out.double().cpu() / 16, ref / 16, **F16TOL)


def test_tc_config2_shape_spot_check():
    b, c, h, w, levels, r = 2, 256, 135, 240, 4, 4
    f1, f2, co, fm1, packed = _inputs(b, c, h, w, levels, "gauss_oob", seed=8)
    co16 = co.half()
    out = ops.pyramid_corr_forward(fm1, packed, co16.to(DEV), r, levels, 1, False,
                                   1.0 / 16, _lib.ENGINE_TC)
    g = torch.Generator().manual_seed(3)
    n = 400
    pts = torch.stack([torch.randint(0, b, (n,), generator=g), torch.randint(0, h, (n,), generator=g),
                       torch.randint(0, w, (n,), generator=g)], 1)
    ref = oracle.pyramid_corr_points(f1.float(), f2.float(), co16.float(), levels, r, pts)
    got = out.float().cpu()[pts[:, 0], :, :, pts[:, 1], pts[:, 2]]
    torch.testing.assert_close(got.double(), ref / 16, **F16TOL)
    simt = ops.pyramid_corr_forward(fm1, packed, co16.to(DEV), r, levels, 1, False, 1.0 / 16,
                                    _lib.ENGINE_SIMT)
    torch.testing.assert_close(out.float(), simt.float(), rtol=2e-3, atol=2e-3)


BWD_CASES = [
    (2, 256, 40, 52, 4, 4, "gauss_oob"),
    (1, 128, 33, 70, 4, 3, "smooth"),
    (1, 128, 30, 40, 4, 8, "uniform64"),
    (1, 64, 24, 36, 2, 4, "uniform8"),
    (1, 256, 24, 40, 3, 3, "converge"),
]


@pytest.mark.parametrize("case", BWD_CASES, ids=lambda c: "b{}c{}_{}x{}_l{}r{}_{}".format(*c))
def test_tc_backward_vs_oracle_and_simt(case):
    b, c, h, w, levels, r, kind = case
    f1, f2, co, fm1, packed = _inputs(b, c, h, w, levels, kind, seed=11)
    co16 = co.half()
    rd = 2 * r + 1
    scale = 1.0 / math.sqrt(c)
    gout = torch.randn(b, levels, rd * rd, h, w, generator=torch.Generator().manual_seed(4)).half()
    g1, g2 = ops.pyramid_corr_backward(fm1, packed, co16.to(DEV), gout.to(DEV), r, levels, 1,
                                       False, scale, _lib.ENGINE_TC)
    s1, s2 = ops.pyramid_corr_backward(fm1, packed, co16.to(DEV), gout.to(DEV), r, levels, 1,
                                       False, scale, _lib.ENGINE_SIMT)
    torch.testing.assert_close(g1.float(), s1.float(), rtol=1e-2, atol=1e-2)
    torch.testing.assert_close(g2, s2, rtol=1e-2, atol=1e-2)
    # oracle: gradients of the (scaled) pyramid correlation w.r.t. the NHWC
    # fmap1 and the NCHW fmap2 (through the pyramid build's gradient)
    x1 = f1.double().requires_grad_(True)
    x2 = f2.double().requires_grad_(True)
    o = oracle.pyramid_corr(x1, x2, co16.double(), levels, r) * scale
    e1, e2 = torch.autograd.grad(o, [x1, x2], gout.double())
    torch.testing.assert_close(g1.permute(0, 3, 1, 2).double().cpu(), e1, **F16TOL)
    g2n = ops.pyramid_build_backward(g2, (b, c, h, w), levels, torch.float32)
    torch.testing.assert_close(g2n.double().cpu(), e2, rtol=1e-2, atol=1e-2)


def test_tc_backward_accumulates_into_reference_buffer():
    # launchLocalCorrCudaPyramidBackward adds into the caller's float32 buffer.
    import localcorr_b200 as lc

    b, c, h, w, levels, r = 1, 128, 30, 44, 4, 4
    f1, f2, co, fm1, packed = _inputs(b, c, h, w, levels, "gauss_oob", seed=12)
    fm1 = fm1.requires_grad_(True)
    packed = packed.requires_grad_(True)
    out = lc.LocalCorrCudaPyramidFunction.apply(fm1, packed, co.half().to(DEV), r, levels, 1,
                                                False)
    g = torch.randn(out.shape, generator=torch.Generator().manual_seed(5)).half().to(DEV)
    a1, a2 = torch.autograd.grad(out, [fm1, packed], g)
    s1, s2 = ops.pyramid_corr_backward(fm1.detach(), packed.detach(), co.half().to(DEV), g, r,
                                       levels, 1, False, 1.0, _lib.ENGINE_SIMT)
    torch.testing.assert_close(a1.float(), s1.float(), rtol=1e-2, atol=2e-2)
    torch.testing.assert_close(a2.float(), s2.half().float(), rtol=1e-2, atol=2e-2)


def test_tc_backward_config2_shape_adjoint():
    # <grad_f1, d1> == <g, corr(d1, f2)> and <grad_f2, d2> == <g, corr(f1, d2)>
    # at the full configuration-2 image size (one image), float16 engine.
    b, c, h, w, levels, r = 1, 256, 135, 240, 4, 4
    f1, f2, co, fm1, packed = _inputs(b, c, h, w, levels, "gauss_oob", seed=13)
    co16 = co.half().to(DEV)
    g = (torch.randn(b, levels, 81, h, w, generator=torch.Generator().manual_seed(6)) * 0.25).half().to(DEV)
    g1, g2 = ops.pyramid_corr_backward(fm1, packed, co16, g, r, levels, 1, False, 1.0 / 16,
                                       _lib.ENGINE_TC)
    d1 = (torch.randn(fm1.shape, generator=torch.Generator().manual_seed(7)) * 0.5).half().to(DEV)
    d2 = (torch.randn(packed.shape, generator=torch.Generator().manual_seed(8)) * 0.5).half().to(DEV)
    c1 = ops.pyramid_corr_forward(d1, packed, co16, r, levels, 1, False, 1.0 / 16, _lib.ENGINE_TC)
    c2 = ops.pyramid_corr_forward(fm1, d2, co16, r, levels, 1, False, 1.0 / 16, _lib.ENGINE_TC)
    lhs1 = (g1.double() * d1.double()).sum().item()
    rhs1 = (g.double() * c1.double()).sum().item()
    lhs2 = (g2.double() * d2.double()).sum().item()
    rhs2 = (g.double() * c2.double()).sum().item()
    assert abs(lhs1 - rhs1) <= 2e-3 * (abs(rhs1) + (g.double().norm() * c1.double().norm()).item() * 1e-2)
    assert abs(lhs2 - rhs2) <= 2e-3 * (abs(rhs2) + (g.double().norm() * c2.double().norm()).item() * 1e-2)


def test_reference_abi_scratch_alternating_streams():
    # The reference-compatible launcher takes no workspace; its library
    # scratch is one buffer per device. Calls alternate between two streams
    # with growing (then shrinking) shapes, so the buffer is regrown while
    # the other stream's call may still run; each call still matches the
    # oracle.
    lib = _lib.load_library()
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    shapes = [(1, 128, 24, 40), (2, 128, 48, 64), (2, 256, 64, 96), (1, 128, 30, 44),
              (2, 256, 72, 100)]
    runs = []
    for i, (b, c, h, w) in enumerate(shapes):
        f1, f2, co, fm1, packed = _inputs(b, c, h, w, 4, "gauss_oob", seed=70 + i)
        co16 = co.half()
        cod = co16.to(DEV)
        out = torch.empty((b, 4, 81, h, w), dtype=torch.float16, device=DEV)
        st = streams[i % 2]
        st.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(st):
            ok = lib.launchLocalCorrCudaPyramidForward(
                fm1.data_ptr(), packed.data_ptr(), cod.data_ptr(), out.data_ptr(), b, h, w, c,
                4, 4, 1, True, False, st.cuda_stream)
        assert ok, _lib.last_error(lib)
        runs.append((f1, f2, co16, fm1, packed, cod, out))
    torch.cuda.synchronize()
    for f1, f2, co16, _, _, _, out in runs:
        c = f1.shape[1]
        ref = oracle.pyramid_corr(f1.float(), f2.float(), co16.float(), 4, 4)
        s = 1.0 / math.sqrt(c)
        torch.testing.assert_close(out.double().cpu() * s, ref * s, **F16TOL)


def test_backward_reuses_the_forward_sort():
    # ...ForwardKeepSort leaves the pixel sort in a caller buffer and
    # ...BackwardWithSort uses it instead of sorting again: same outputs and
    # gradients as the self-sorting calls (grad_fmap2 up to the float32
    # order of the reductions), and the backward launches no sort kernels.
    lib = _lib.load_library()
    b, c, h, w, levels, r = 2, 256, 40, 52, 4, 4
    f1, f2, co, fm1, packed = _inputs(b, c, h, w, levels, "gauss_oob", seed=21)
    cod = co.half().to(DEV)
    nb = ops.sort_state_bytes(fm1, packed, r, levels, engine=_lib.ENGINE_TC)
    assert 0 < nb < 16 << 20
    ss = torch.empty(nb, dtype=torch.uint8, device=DEV)
    out_k = ops.pyramid_corr_forward(fm1, packed, cod, r, levels, 1, False, 0.0625,
                                     _lib.ENGINE_TC, sort_state=ss)
    out_r = ops.pyramid_corr_forward(fm1, packed, cod, r, levels, 1, False, 0.0625,
                                     _lib.ENGINE_TC)
    assert torch.equal(out_k, out_r)
    gout = torch.randn(out_r.shape, generator=torch.Generator().manual_seed(22)).half().to(DEV)
    torch.cuda.synchronize()
    lib.localCorrB200LaunchCount(1)
    g1a, g2a = ops.pyramid_corr_backward(fm1, packed, cod, gout, r, levels, 1, False, 0.0625,
                                         _lib.ENGINE_TC, sort_state=ss)
    n_with = lib.localCorrB200LaunchCount(1)
    g1b, g2b = ops.pyramid_corr_backward(fm1, packed, cod, gout, r, levels, 1, False, 0.0625,
                                         _lib.ENGINE_TC)
    n_without = lib.localCorrB200LaunchCount(1)
    torch.cuda.synchronize()
    # the sort's launches: histogram fused with the scan + scatter for small
    # problems, else histogram + three scan passes + scatter
    assert n_without - n_with in (2, 5)
    assert torch.equal(g1a, g1b)
    torch.testing.assert_close(g2a, g2b, rtol=1e-5, atol=1e-5)
    # and against the oracle
    x1 = f1.double().requires_grad_(True)
    x2 = f2.double().requires_grad_(True)
    o = oracle.pyramid_corr(x1, x2, co.half().double(), levels, r) * 0.0625
    e1, e2 = torch.autograd.grad(o, [x1, x2], gout.double().cpu())
    torch.testing.assert_close(g1a.permute(0, 3, 1, 2).double().cpu(), e1, **F16TOL)
    g2n = ops.pyramid_build_backward(g2a, (b, c, h, w), levels, torch.float32)
    torch.testing.assert_close(g2n.double().cpu(), e2, **F16TOL)


def test_sort_state_too_small_is_rejected():
    lib = _lib.load_library()
    b, c, h, w, levels, r = 1, 128, 24, 40, 4, 4
    f1, f2, co, fm1, packed = _inputs(b, c, h, w, levels, "uniform8", seed=23)
    nb = ops.sort_state_bytes(fm1, packed, r, levels, engine=_lib.ENGINE_TC)
    ss = torch.empty(nb - 256, dtype=torch.uint8, device=DEV)
    with pytest.raises(RuntimeError, match="sort state too small"):
        ops.pyramid_corr_forward(fm1, packed, co.half().to(DEV), r, levels, 1, False, 1.0,
                                 _lib.ENGINE_TC, sort_state=ss)
    assert lib.localCorrB200PyramidSortStateBytes(1, 24, 40, 24, 40, 128, 4, 4, 1, _lib.F32,
                                                  _lib.ENGINE_AUTO) == 0
