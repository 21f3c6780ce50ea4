"""CUDA engine parity against the CPU oracle and the reference's golden fixtures.

Tolerances (the parity contract): float32 rtol 1e-5 / atol 1e-4; float16
rtol 1e-2 / atol 1e-2 against a float64 oracle evaluated on the same
float16-rounded inputs. Every case runs through the C ABI (ctypes) of the
built library; both engines are exercised where they apply.
"""

import math
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import localcorr_b200 as lc
from localcorr_b200 import _lib, ops
from oracle import oracle

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
DEV = "cuda"
TOL = {torch.float32: dict(rtol=1e-5, atol=1e-4), torch.float16: dict(rtol=1e-2, atol=1e-2)}


@pytest.fixture(scope="module", autouse=True)
def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    lib = _lib.load_library()
    assert lib is not None, "liblocalcorr_b200.so must be built for the GPU tests"


def _t(a, dtype=torch.float32):
    return torch.from_numpy(np.asarray(a)).to(dtype)


def _close(actual, expected, dtype):
    torch.testing.assert_close(actual.double().cpu(), expected.double().cpu(), **TOL[dtype])


def _engines():
    return [_lib.ENGINE_SIMT, _lib.ENGINE_AUTO]


# ---------------------------------------------------------------------------
# golden fixtures (outputs of the reference itself)
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("path", sorted(GOLDEN.glob("pyr_*.npz")), ids=lambda p: p.stem)
def test_block_matches_reference_golden(path):
    d = np.load(path)
    levels, radius = int(d["levels"]), int(d["radius"])
    f1 = _t(d["fmap1"]).to(DEV).requires_grad_(True)
    f2 = _t(d["fmap2"]).to(DEV).requires_grad_(True)
    coords = _t(d["coords"]).to(DEV)
    b, c, h, w = f1.shape
    block = lc.get_localcorr_block(f1, f2, num_levels=levels, radius=radius,
                                   corr_mode="localcorr_cuda")
    out = block(coords)
    ref = _t(d["out_ref"]).reshape(b, -1, h, w) / math.sqrt(c)
    _close(out.detach(), ref, torch.float32)
    out.backward(_t(d["grad_out"]).to(DEV))
    _close(f1.grad, _t(d["grad_fmap1"]), torch.float32)
    _close(f2.grad, _t(d["grad_fmap2"]), torch.float32)


def test_dilated_ymajor_matches_reference_golden():
    d = np.load(GOLDEN / "dil_b1c6_12x14_r3d2.npz")
    r, dil = int(d["radius"]), int(d["dilation"])
    f1, f2 = _t(d["fmap1"]).to(DEV), _t(d["fmap2"]).to(DEV)
    ref = _t(d["out_ref"])
    # Pyramid engine, one level, identity coords, y-major.
    b, c, h, w = f1.shape
    fm1 = f1.permute(0, 2, 3, 1).contiguous()
    packed = f2.permute(0, 2, 3, 1).contiguous().reshape(b, -1)
    grid = ops.identity_coords(b, h, w, torch.float32, f1.device)
    out = lc.LocalCorrCudaPyramidFunction.apply(fm1, packed, grid, r, 1, dil, True)
    _close(out.reshape(ref.shape), ref, torch.float32)
    # Spatial kernel with dilation.
    blk = lc.LocalCorrCudaPyramidSpatialBlock(f1, f2, radius=r, dilation=dil, normalize=None)
    _close(blk(), ref, torch.float32)


@pytest.mark.parametrize("path", sorted(GOLDEN.glob("spatial_*.npz")), ids=lambda p: p.stem)
def test_sampler_matches_reference_golden(path):
    d = np.load(path)
    r = int(d["radius"])
    i1 = _t(d["in1"]).to(DEV).requires_grad_(True)
    i2 = _t(d["in2"]).to(DEV).requires_grad_(True)
    sampler = lc.get_localcorr_sampler(patch_size=2 * r + 1, corr_mode="localcorr_cuda")
    out = sampler(i1, i2)
    _close(out.detach(), _t(d["out_ref"]), torch.float32)
    out.backward(_t(d["grad_out"]).to(DEV))
    _close(i1.grad, _t(d["grad_in1"]), torch.float32)
    _close(i2.grad, _t(d["grad_in2"]), torch.float32)


# ---------------------------------------------------------------------------
# oracle sweeps
# ---------------------------------------------------------------------------

PYR_CASES = [
    # B, C, H, W, L, r, max_disp
    (2, 64, 40, 52, 4, 4, 8.0),   # reference GPU test shape (tests/test_cuda_kernels.py:27-28)
    (1, 256, 46, 62, 4, 4, 8.0),  # benchmark configuration 1 shape
    (2, 48, 23, 31, 3, 3, 6.0),   # C not a multiple of 32, odd dims
    (1, 196, 14, 18, 1, 4, 3.0),  # PWC level channel count
    (1, 3, 9, 11, 2, 1, 2.0),     # tiny C
    (1, 32, 20, 24, 2, 0, 2.0),   # radius 0
    (1, 128, 16, 32, 4, 8, 20.0), # radius 8 (configuration 5)
    (2, 16, 64, 40, 5, 2, 4.0),   # 5 levels (beyond the fused pyramid build)
]


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16], ids=["f32", "f16"])
@pytest.mark.parametrize("case", PYR_CASES, ids=lambda c: "b{}c{}_{}x{}_l{}r{}".format(*c[:6]))
def test_block_forward_backward_vs_oracle(case, dtype):
    b, c, h, w, levels, radius, md = case
    f1, f2 = oracle.make_fmaps(b, c, h, w, seed=c + h)
    coords = oracle.make_coords_uniform(b, h, w, md, seed=w)
    if dtype == torch.float16:
        f1, f2, coords = f1.half().float(), f2.half().float(), coords.half().float()
    g = torch.Generator().manual_seed(5)
    rd = 2 * radius + 1
    grad_out = torch.randn(b, levels * rd * rd, h, w, generator=g)
    if dtype == torch.float16:
        grad_out = grad_out.half().float()
    ref_out, ref_g1, ref_g2 = oracle.block_grads(f1, f2, coords, levels, radius, grad_out)
    x1 = f1.to(DEV, dtype).requires_grad_(True)
    x2 = f2.to(DEV, dtype).requires_grad_(True)
    block = lc.get_localcorr_block(x1, x2, num_levels=levels, radius=radius)
    out = block(coords.to(DEV, dtype))
    assert out.dtype == dtype and out.shape == (b, levels * rd * rd, h, w)
    _close(out.detach(), ref_out, dtype)
    out.backward(grad_out.to(DEV, dtype))
    assert x1.grad.dtype == dtype and x2.grad.dtype == dtype
    _close(x1.grad, ref_g1, dtype)
    _close(x2.grad, ref_g2, dtype)


@pytest.mark.parametrize("engine", _engines(), ids=["simt", "auto"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16], ids=["f32", "f16"])
@pytest.mark.parametrize("dil,ymajor", [(1, False), (1, True), (2, True), (3, False)])
def test_extended_abi_engines_dilation_ymajor(engine, dtype, dil, ymajor):
    b, c, h, w, levels, radius = 1, 40, 18, 22, 2, 2
    f1, f2 = oracle.make_fmaps(b, c, h, w, seed=3)
    coords = oracle.make_coords_uniform(b, h, w, 4.0, seed=4)
    if dtype == torch.float16:
        f1, f2, coords = f1.half().float(), f2.half().float(), coords.half().float()
    ref = oracle.pyramid_corr(f1, f2, coords, levels, radius, dilation=dil, ymajor=ymajor)
    fm1 = ops.nchw_to_nhwc(f1.to(DEV, dtype))
    packed = ops.pyramid_build(f2.to(DEV, dtype), levels)
    out = ops.pyramid_corr_forward(fm1, packed, coords.to(DEV, dtype), radius, levels, dil,
                                   ymajor, 0.5, engine)
    _close(out, ref * 0.5, dtype)
    # Backward through the same ABI: check against the oracle's autograd.
    g = torch.randn(out.shape, generator=torch.Generator().manual_seed(9))
    if dtype == torch.float16:
        g = g.half().float()
    x1 = f1.double().requires_grad_(True)
    x2 = f2.double().requires_grad_(True)
    o = oracle.pyramid_corr(x1, x2, coords, levels, radius, dilation=dil, ymajor=ymajor) * 0.5
    e1, e2 = torch.autograd.grad(o, [x1, x2], g.double())
    g1, g2p = ops.pyramid_corr_backward(fm1, packed, coords.to(DEV, dtype), g.to(DEV, dtype),
                                        radius, levels, dil, ymajor, 0.5, engine)
    g2 = ops.pyramid_build_backward(g2p, (b, c, h, w), levels, dtype)
    _close(g1.permute(0, 3, 1, 2), e1, dtype)
    _close(g2, e2, dtype)


def test_float32_coords_with_float16_maps():
    b, c, h, w = 1, 64, 30, 40
    f1, f2 = oracle.make_fmaps(b, c, h, w, seed=8)
    f1, f2 = f1.half().float(), f2.half().float()
    coords = oracle.make_coords_uniform(b, h, w, 6.0, seed=9) + 300.0 * 0  # fp32 precision kept
    ref = oracle.block_forward(f1, f2, coords, 3, 3)
    block = lc.get_localcorr_block(f1.to(DEV).half(), f2.to(DEV).half(), 3, 3)
    _close(block(coords.to(DEV)), ref, torch.float16)


# ---------------------------------------------------------------------------
# reference-compatible Function and C ABI behaviour
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("levels,radius", [(1, 4), (2, 2), (3, 3), (4, 4)])
def test_reference_function_matches_oracle(levels, radius):
    # tests/test_cuda_kernels.py:133-158 of the reference, through the
    # reference-compatible launchers.
    b, c, h, w = 2, 64, 40, 52
    f1, f2 = oracle.make_fmaps(b, c, h, w, seed=60)
    coords = oracle.make_coords_uniform(b, h, w, 2.0, seed=61)
    fm1 = f1.permute(0, 2, 3, 1).contiguous().to(DEV).requires_grad_(True)
    pyr = oracle.build_pyramid(f2, levels)
    packed = torch.cat([p.permute(0, 2, 3, 1).reshape(b, -1) for p in pyr], 1).contiguous()
    packed = packed.to(DEV).requires_grad_(True)
    co = coords.to(DEV).requires_grad_(True)
    out = lc.LocalCorrCudaPyramidFunction.apply(fm1, packed, co, radius, levels, 1, False)
    ref = oracle.pyramid_corr(f1, f2, coords, levels, radius)
    _close(out.detach(), ref, torch.float32)
    g = torch.randn(out.shape, generator=torch.Generator().manual_seed(2))
    gf1, gp, gc = torch.autograd.grad(out, [fm1, packed, co], g.to(DEV))
    assert gc.abs().sum().item() == 0.0
    x1 = f1.double().requires_grad_(True)
    xp = [p.double().detach().requires_grad_(True) for p in pyr]
    # oracle on the packed levels directly: gradient w.r.t. each level
    o = _oracle_on_levels(x1, xp, coords, radius)
    e1, *ep = torch.autograd.grad(o, [x1, *xp], g.double())
    _close(gf1.permute(0, 3, 1, 2), e1, torch.float32)
    ep_packed = torch.cat([e.permute(0, 2, 3, 1).reshape(b, -1) for e in ep], 1)
    _close(gp, ep_packed, torch.float32)


def _oracle_on_levels(f1, levels_nchw, coords, radius):
    """pyramid_corr with the level maps given (no pooling)."""
    outs = []
    for lvl, f2l in enumerate(levels_nchw):
        # Scale coords so that level lvl sees coords / 2^lvl: run a one-level
        # oracle on pre-scaled coordinates.
        co = coords.double() / float(2 ** lvl)
        outs.append(oracle.pyramid_corr(f1, f2l, co, 1, radius)[:, 0])
    return torch.stack(outs, 1)


def test_reference_function_half_grads_dtype():
    b, c, h, w = 2, 64, 40, 52
    f1, f2 = oracle.make_fmaps(b, c, h, w, seed=64)
    coords = oracle.make_coords_uniform(b, h, w, 2.0, seed=65)
    f1h = f1.half().to(DEV).requires_grad_(True)
    f2h = f2.half().to(DEV).requires_grad_(True)
    block = lc.get_localcorr_block(f1h, f2h, num_levels=3, radius=3, corr_mode="localcorr_cuda")
    out = block(coords.half().to(DEV))
    (out * torch.randn_like(out)).sum().backward()
    assert f1h.grad.dtype == torch.float16 and f2h.grad.dtype == torch.float16
    assert torch.isfinite(f1h.grad).all() and torch.isfinite(f2h.grad).all()


def test_coords_grad_is_zero():
    f1, f2 = oracle.make_fmaps(2, 16, 20, 24, seed=68)
    coords = oracle.make_coords_uniform(2, 20, 24, 2.0).to(DEV).requires_grad_(True)
    block = lc.get_localcorr_block(f1.to(DEV), f2.to(DEV), num_levels=2, radius=2)
    block(coords).square().mean().backward()
    assert coords.grad is not None and coords.grad.abs().sum().item() == 0.0


def test_reference_helper_guards():
    from localcorr_b200.blocks import _localcorr_cuda_pyramid_forward

    f = torch.zeros(1, 8, 8, 4, device=DEV)
    p = torch.zeros(1, 4 * 64, device=DEV)
    with pytest.raises(RuntimeError, match="coords dtype"):
        _localcorr_cuda_pyramid_forward(f, p, torch.zeros(1, 2, 8, 8, device=DEV).half(), 1, 1)
    with pytest.raises(RuntimeError, match="float32 or float16"):
        _localcorr_cuda_pyramid_forward(f.bfloat16(), p.bfloat16(),
                                        torch.zeros(1, 2, 8, 8, device=DEV).bfloat16(), 1, 1)


def test_invalid_launch_raises_runtime_error():
    f = torch.zeros(1, 8, 8, 4, device=DEV)
    p = torch.zeros(1, 4 * 64, device=DEV)
    co = torch.zeros(1, 2, 8, 8, device=DEV)
    with pytest.raises(RuntimeError, match="levels"):
        lc.LocalCorrCudaPyramidFunction.apply(f, p, co, 1, 9, 1, False)


def test_far_outside_coords_exact_zeros_and_no_grad():
    f1, f2 = oracle.make_fmaps(1, 32, 16, 24, seed=13)
    x1, x2 = f1.to(DEV).requires_grad_(True), f2.to(DEV).requires_grad_(True)
    block = lc.get_localcorr_block(x1, x2, num_levels=3, radius=2)
    out = block(torch.full((1, 2, 16, 24), 1000.0, device=DEV))
    assert torch.count_nonzero(out) == 0
    out.sum().backward()
    assert x1.grad.abs().sum() == 0 and x2.grad.abs().sum() == 0


# ---------------------------------------------------------------------------
# layout kernels
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("dtype", [torch.float32, torch.float16], ids=["f32", "f16"])
@pytest.mark.parametrize("shape,levels", [((2, 40, 37, 70), 4), ((1, 8, 135, 240), 4),
                                          ((1, 5, 300, 70), 6)])
def test_pyramid_build_matches_torch_chain(shape, levels, dtype):
    x = torch.randn(shape, generator=torch.Generator().manual_seed(1)).to(DEV, dtype)
    packed = ops.pyramid_build(x, levels)
    pyr = [x]
    for _ in range(1, levels):
        pyr.append(F.avg_pool2d(pyr[-1], 2, stride=2))
    ref = torch.cat([p.permute(0, 2, 3, 1).reshape(shape[0], -1) for p in pyr], 1)
    torch.testing.assert_close(packed, ref, rtol=0, atol=0)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16], ids=["f32", "f16"])
def test_pyramid_build_backward_matches_autograd(dtype):
    shape, levels = (2, 24, 45, 66), 4
    x = torch.randn(shape, generator=torch.Generator().manual_seed(2)).to(DEV)
    xr = x.clone().requires_grad_(True)
    pyr = [xr]
    for _ in range(1, levels):
        pyr.append(F.avg_pool2d(pyr[-1], 2, stride=2))
    ref = torch.cat([p.permute(0, 2, 3, 1).reshape(shape[0], -1) for p in pyr], 1)
    g = torch.randn(ref.shape, generator=torch.Generator().manual_seed(3)).to(DEV)
    (eg,) = torch.autograd.grad(ref, [xr], g)
    out = ops.pyramid_build_backward(g, shape, levels, dtype)
    _close(out, eg, dtype)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16], ids=["f32", "f16"])
def test_transposes_exact(dtype):
    x = torch.randn(3, 70, 33, 41, generator=torch.Generator().manual_seed(4)).to(DEV, dtype)
    y = ops.nchw_to_nhwc(x)
    assert torch.equal(y, x.permute(0, 2, 3, 1).contiguous())
    assert torch.equal(ops.nhwc_to_nchw(y), x)


# ---------------------------------------------------------------------------
# spatial (PWC) correlation
# ---------------------------------------------------------------------------

# The first three are configuration-3 levels; W % 4 == 0 with dilation 1
# takes the tiled kernels (radius 1..3 with a halo that is not a whole
# 4-element unit included), the others the general kernels.
SPATIAL_CASES = [(8, 196, 7, 16, 4, 1), (2, 32, 112, 256, 4, 1), (2, 96, 28, 64, 4, 1),
                 (1, 13, 11, 37, 3, 2), (1, 8, 9, 40, 2, 3), (1, 16, 10, 12, 0, 1),
                 (1, 24, 20, 30, 6, 2), (2, 20, 17, 24, 3, 1), (1, 40, 13, 20, 1, 1),
                 (1, 12, 9, 36, 2, 1), (1, 33, 15, 44, 4, 1)]


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16], ids=["f32", "f16"])
@pytest.mark.parametrize("case", SPATIAL_CASES, ids=lambda c: "b{}c{}_{}x{}_r{}d{}".format(*c))
def test_spatial_vs_oracle(case, dtype):
    b, c, h, w, r, dil = case
    i1, i2 = oracle.make_fmaps(b, c, h, w, seed=h)
    if dtype == torch.float16:
        i1, i2 = i1.half().float(), i2.half().float()
    g = torch.randn(b, 2 * r + 1, 2 * r + 1, h, w, generator=torch.Generator().manual_seed(1))
    if dtype == torch.float16:
        g = g.half().float()
    ref, e1, e2 = oracle.spatial_grads(i1, i2, r, g, dilation=dil)
    x1 = i1.to(DEV, dtype).requires_grad_(True)
    x2 = i2.to(DEV, dtype).requires_grad_(True)
    out = ops.spatial_corr(x1, x2, r, dil, 1.0)
    _close(out.detach(), ref, dtype)
    out.backward(g.to(DEV, dtype))
    _close(x1.grad, e1, dtype)
    _close(x2.grad, e2, dtype)


def test_pyramid_sampler_module():
    i1, i2 = oracle.make_fmaps(2, 32, 24, 30, seed=42)
    s = lc.LocalCorrCudaPyramidSampler(patch_size=9)
    out = s(i1.to(DEV), i2.to(DEV))
    _close(out, oracle.spatial_corr(i1, i2, 4), torch.float32)


# ---------------------------------------------------------------------------
# full benchmark sizes: spot checks and size-independent properties
# ---------------------------------------------------------------------------

def test_config2_shape_spot_check_and_adjoint():
    b, c, h, w, levels, radius = 1, 256, 135, 240, 4, 4
    f1, f2 = oracle.make_fmaps(b, c, h, w, seed=2)
    coords = oracle.make_coords_gauss_oob(b, h, w, 6.0, 0.05, seed=3)
    f1h, f2h, coh = f1.half(), f2.half(), coords.half()
    x1 = f1h.to(DEV).requires_grad_(True)
    x2 = f2h.to(DEV).requires_grad_(True)
    block = lc.get_localcorr_block(x1, x2, levels, radius)
    out = block(coh.to(DEV))
    pts = torch.stack([torch.zeros(300, dtype=torch.long),
                       torch.randint(0, h, (300,), generator=torch.Generator().manual_seed(1)),
                       torch.randint(0, w, (300,), generator=torch.Generator().manual_seed(2))], 1)
    ref = oracle.pyramid_corr_points(f1h.float(), f2h.float(), coh.float(), levels, radius, pts)
    got = out.detach().float().cpu().reshape(b, levels, 81, h, w)[pts[:, 0], :, :, pts[:, 1],
                                                                   pts[:, 2]]
    _close(got, ref / math.sqrt(c), torch.float16)
    # Adjoint identity (corr is linear in each map): <dL/df1, d1> equals
    # <grad_out, corr(d1, f2)>, checked in float32 at full size.
    f1d, f2d = x1.detach().float(), x2.detach().float()
    co32 = coh.float().to(DEV)
    go = torch.randn(out.shape, generator=torch.Generator().manual_seed(7)).to(DEV)
    a1 = f1d.clone().requires_grad_(True)
    a2 = f2d.clone().requires_grad_(True)
    o32 = lc.get_localcorr_block(a1, a2, levels, radius)(co32)
    o32.backward(go)
    d1 = torch.randn_like(f1d)
    d2 = torch.randn_like(f2d)
    lhs1 = (a1.grad.double() * d1.double()).sum()
    rhs1 = (go.double() * lc.get_localcorr_block(d1, f2d, levels, radius)(co32).double()).sum()
    lhs2 = (a2.grad.double() * d2.double()).sum()
    rhs2 = (go.double() * lc.get_localcorr_block(f1d, d2, levels, radius)(co32).double()).sum()
    assert abs((lhs1 - rhs1).item()) <= 1e-4 * abs(rhs1.item()) + 1e-2
    assert abs((lhs2 - rhs2).item()) <= 1e-4 * abs(rhs2.item()) + 1e-2
