"""Parity at the benchmark configurations' own sizes, through the C ABI.

The dense float64 oracle is too slow for 135x240 frames at B>1, so these
checks compare the engine with the point-subset oracles (outputs at sampled
pixels, fmap1 gradients at sampled pixels, pyramid-level gradients at
sampled level positions), all pinned to the reference's own fixtures on the
CPU (tests/test_oracle_golden.py). Tolerances are the parity contract's:
float16 rtol 1e-2 / atol 1e-2 against the oracle on the same float16 inputs.

* configuration 2: B=2 of the 135x240, C=256, L=4, r=4 training frames,
  Gaussian flow with 5% far out-of-bounds pixels, tensor-core engine,
  forward and both gradients;
* configuration 4: one 270x480 frame, smooth flow, forward, whole frame and
  as row bands through the map-size entry points and the row-band block;
* configuration 5: B=8, C=128, 64x128, U(-1,1) maps, U(-64,64) flow (heavy
  zero padding, crowded coarse levels), r in {3, 4, 8}, forward and both
  gradients;
* small incoming gradients (x 1e-4): the float16 gradient records keep the
  gradient's own magnitude (the output scale is applied in float32), so
  their relative error stays at float16 rounding.
"""

import math

import pytest
import torch

import localcorr_b200 as lc
from localcorr_b200 import _lib, bands, ops
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


def _pixels(b, h, w, n, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.stack([torch.randint(0, b, (n,), generator=g),
                        torch.randint(0, h, (n,), generator=g),
                        torch.randint(0, w, (n,), generator=g)], 1)


def _level_positions(b, h, w, levels, n_per_level, seed):
    g = torch.Generator().manual_seed(seed)
    rows = []
    for lvl in range(levels):
        hl, wl = h >> lvl, w >> lvl
        rows.append(torch.stack([torch.randint(0, b, (n_per_level,), generator=g),
                                 torch.full((n_per_level,), lvl),
                                 torch.randint(0, hl, (n_per_level,), generator=g),
                                 torch.randint(0, wl, (n_per_level,), generator=g)], 1))
    return torch.cat(rows)


def _packed_at(g2, pos, c, h, w, levels):
    """Rows of the packed [B, C*sum h_l w_l] gradient at (b, l, y, x)."""
    offs = [0]
    for lvl in range(levels):
        offs.append(offs[-1] + c * (h >> lvl) * (w >> lvl))
    idx = [offs[l] + (y * (w >> l) + x) * c for _, l, y, x in pos.tolist()]
    rows = torch.stack([g2[b, i:i + c] for (b, _, _, _), i in zip(pos.tolist(), idx)])
    return rows.double().cpu()


def _check_case(f1, f2, co16, gout16, levels, r, n_pix, n_pos, seed, engine=_lib.ENGINE_TC,
                gscale=1.0):
    """Forward at n_pix pixels, grad fmap1 at n_pix pixels, level gradients
    at n_pos positions per level; gout16 is the float16 incoming gradient
    and gscale a factor the comparison divides out of both sides."""
    b, c, h, w = f1.shape
    scale = 1.0 / math.sqrt(c)
    fm1 = ops.nchw_to_nhwc(f1.to(DEV))
    packed = ops.pyramid_build(f2.to(DEV), levels)
    cod = co16.to(DEV)
    out = ops.pyramid_corr_forward(fm1, packed, cod, r, levels, 1, False, scale, engine)
    pts = _pixels(b, h, w, n_pix, seed)
    f1d, f2d, cod64 = f1.double(), f2.double(), co16.double()
    ref = oracle.pyramid_corr_points(f1d, f2d, cod64, levels, r, pts) * scale
    got = out.double().cpu()[pts[:, 0], :, :, pts[:, 1], pts[:, 2]]
    torch.testing.assert_close(got, ref, **F16TOL)
    g1, g2 = ops.pyramid_corr_backward(fm1, packed, cod, gout16.to(DEV), r, levels, 1, False,
                                       scale, engine)
    go64 = gout16.double()
    e1 = oracle.pyramid_corr_points_grad_fmap1(f1d, f2d, cod64, levels, r, pts, go64) * scale
    got1 = g1.double().cpu()[pts[:, 0], pts[:, 1], pts[:, 2]]
    torch.testing.assert_close(got1 / gscale, e1 / gscale, **F16TOL)
    pos = _level_positions(b, h, w, levels, n_pos, seed + 1)
    e2 = oracle.pyramid_corr_points_grad_levels(f1d, f2d, cod64, levels, r, pos, go64) * scale
    got2 = _packed_at(g2, pos, c, h, w, levels)
    torch.testing.assert_close(got2 / gscale, e2 / gscale, **F16TOL)
    return out, g1, g2


def test_config2_training_frames_tc_forward_and_gradients():
    b, c, h, w, levels, r = 2, 256, 135, 240, 4, 4
    f1, f2 = oracle.make_fmaps(b, c, h, w, seed=31)
    f1, f2 = f1.half().float(), f2.half().float()
    co16 = oracle.make_coords_gauss_oob(b, h, w, 6.0, 0.05, seed=32).half()
    gout = torch.randn(b, levels, 81, h, w, generator=torch.Generator().manual_seed(33)).half()
    _check_case(f1.half(), f2.half(), co16, gout, levels, r, n_pix=300, n_pos=75, seed=34)


@pytest.mark.parametrize("r", [3, 4, 8])
def test_config5_highbatch_large_flow(r):
    b, c, h, w, levels = 8, 128, 64, 128, 4
    f1, f2 = oracle.make_fmaps(b, c, h, w, seed=41 + r, dist="uniform")
    co16 = oracle.make_coords_uniform(b, h, w, 64.0, seed=42 + r).half()
    rd = 2 * r + 1
    gout = torch.randn(b, levels, rd * rd, h, w,
                       generator=torch.Generator().manual_seed(43 + r)).half()
    out, g1, g2 = _check_case(f1.half(), f2.half(), co16, gout, levels, r, n_pix=200,
                              n_pos=50, seed=44 + r)
    # whole tensors against the CUDA-core engine (float32 accumulation of the
    # same float16 inputs, atomics instead of the tensor-core pull)
    fm1 = ops.nchw_to_nhwc(f1.half().to(DEV))
    packed = ops.pyramid_build(f2.half().to(DEV), levels)
    scale = 1.0 / math.sqrt(c)
    s_out = ops.pyramid_corr_forward(fm1, packed, co16.to(DEV), r, levels, 1, False, scale,
                                     _lib.ENGINE_SIMT)
    torch.testing.assert_close(out.float(), s_out.float(), rtol=2e-3, atol=2e-3)
    s1, s2 = ops.pyramid_corr_backward(fm1, packed, co16.to(DEV), gout.to(DEV), r, levels, 1,
                                       False, scale, _lib.ENGINE_SIMT)
    torch.testing.assert_close(g1.float(), s1.float(), **F16TOL)
    torch.testing.assert_close(g2, s2, **F16TOL)


def test_small_incoming_gradients_keep_relative_precision():
    b, c, h, w, levels, r = 1, 256, 135, 240, 4, 4
    f1, f2 = oracle.make_fmaps(b, c, h, w, seed=51)
    co16 = oracle.make_coords_gauss_oob(b, h, w, 6.0, 0.05, seed=52).half()
    gs = 1e-4
    gout = (torch.randn(b, levels, 81, h, w, generator=torch.Generator().manual_seed(53))
            * gs).half()
    _check_case(f1.half(), f2.half(), co16, gout, levels, r, n_pix=200, n_pos=50, seed=54,
                gscale=gs)


def test_config4_4k_frame_whole_and_row_bands():
    b, c, h, w, levels, r = 1, 256, 270, 480, 4, 4
    f1, f2 = oracle.make_fmaps(b, c, h, w, seed=61)
    f1, f2 = f1.half(), f2.half()
    co16 = oracle.make_coords_smooth(b, h, w, 40.0, seed=62).half()
    scale = 1.0 / math.sqrt(c)
    fm1 = ops.nchw_to_nhwc(f1.to(DEV))
    packed = ops.pyramid_build(f2.to(DEV), levels)
    cod = co16.to(DEV)
    whole = ops.pyramid_corr_forward(fm1, packed, cod, r, levels, 1, False, scale,
                                     _lib.ENGINE_TC)
    pts = _pixels(b, h, w, 300, 63)
    ref = oracle.pyramid_corr_points(f1.double(), f2.double(), co16.double(), levels, r,
                                     pts) * scale
    got = whole.double().cpu()[pts[:, 0], :, :, pts[:, 1], pts[:, 2]]
    torch.testing.assert_close(got, ref, **F16TOL)
    # row bands of 2, 4 and 8 ranks through the map-size entry points
    for parts in (2, 4, 8):
        outs = []
        for y0, y1 in bands.band_rows(h, parts, 1 << (levels - 1)):
            outs.append(ops.pyramid_corr_forward(
                fm1[:, y0:y1].contiguous(), packed, cod[:, :, y0:y1].contiguous(), r, levels,
                1, False, scale, _lib.ENGINE_TC, map_hw=(h, w)))
        assert torch.equal(torch.cat(outs, dim=3), whole), parts
    # the row-band block on one rank (no process group) is the frame's block
    f1d, f2d = f1.to(DEV), f2.to(DEV)
    with torch.no_grad():
        blk = bands.LocalCorrRowBandBlock(f1d, f2d, h, num_levels=levels, radius=r)
        got_blk = blk(cod)
        want_blk = lc.get_localcorr_block(f1d, f2d, levels, r, corr_mode="localcorr_cuda")(cod)
    assert torch.equal(got_blk, want_blk)
    assert torch.equal(want_blk, whole.reshape(b, -1, h, w))
