"""Row bands of one frame on the GPU: the map-size-decoupled entry points
(``...MapDims``) against the float64 oracle, band outputs against the whole
frame's, band pyramids against the whole frame's pyramid, and the row-band
block on one process and (given two GPUs) on two NCCL ranks.

Tolerances: float16 maps, rtol 1e-2 / atol 1e-2 against the oracle on the same
float16 inputs; float32 maps (CUDA-core engine) rtol/atol 1e-4. A band's rows
of the whole-frame output are computed by the same per-pixel arithmetic, so
band outputs equal the whole frame's rows exactly.
"""

import math
import os
import socket

import pytest
import torch

import localcorr_b200 as lc
from localcorr_b200 import _lib, bands, ops
from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda"
F16TOL = dict(rtol=1e-2, atol=1e-2)
F32TOL = dict(rtol=1e-4, atol=1e-4)


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


def _frame(b, c, h, w, dtype, seed=0, amp=12.0):
    f1, f2 = oracle.make_fmaps(b, c, h, w, seed=seed)
    co = oracle.make_coords_smooth(b, h, w, amp, seed=seed + 1)
    return f1.to(dtype), f2.to(dtype), co.to(dtype)


ENGINES = [(torch.float16, _lib.ENGINE_TC, F16TOL), (torch.float32, _lib.ENGINE_SIMT, F32TOL)]


@pytest.mark.parametrize("dtype,engine,tol", ENGINES, ids=["tc_f16", "simt_f32"])
@pytest.mark.parametrize("rows", [(8, 24), (0, 16), (32, 45), (5, 30)])
def test_map_dims_forward_backward_vs_oracle(dtype, engine, tol, rows):
    b, c, h, w, levels, r = 2, 64, 45, 52, 4, 4
    f1, f2, co = _frame(b, c, h, w, dtype)
    y0, y1 = rows
    f1b, cob = f1[:, :, y0:y1], co[:, :, y0:y1]
    fm1 = ops.nchw_to_nhwc(f1b.to(DEV).contiguous())
    packed = ops.pyramid_build(f2.to(DEV), levels)
    scale = 1.0 / math.sqrt(c)
    out = ops.pyramid_corr_forward(fm1, packed, cob.to(DEV).contiguous(), r, levels,
                                   scale=scale, engine=engine, map_hw=(h, w))
    assert out.shape == (b, levels, (2 * r + 1) ** 2, y1 - y0, w)
    x1 = f1b.double().requires_grad_(True)
    x2 = f2.double().requires_grad_(True)
    ref = oracle.pyramid_corr(x1, x2, cob.double(), levels, r) * scale
    torch.testing.assert_close(out.double().cpu(), ref.detach(), **tol)
    gout = torch.randn(out.shape, generator=torch.Generator().manual_seed(3)).to(dtype)
    g1, g2 = ops.pyramid_corr_backward(fm1, packed, cob.to(DEV).contiguous(), gout.to(DEV), r,
                                       levels, scale=scale, engine=engine, map_hw=(h, w))
    e1, e2 = torch.autograd.grad(ref, [x1, x2], gout.double())
    torch.testing.assert_close(g1.permute(0, 3, 1, 2).double().cpu(), e1, **tol)
    g2n = ops.pyramid_build_backward(g2, (b, c, h, w), levels, torch.float32)
    torch.testing.assert_close(g2n.double().cpu(), e2, **tol)


@pytest.mark.parametrize("dtype,engine", [(torch.float16, _lib.ENGINE_TC),
                                          (torch.float32, _lib.ENGINE_SIMT)],
                         ids=["tc_f16", "simt_f32"])
def test_bands_concatenate_to_the_frame(dtype, engine):
    b, c, h, w, levels, r = 1, 128, 135, 120, 4, 4
    f1, f2, co = _frame(b, c, h, w, dtype, seed=4, amp=40.0)
    fm1 = ops.nchw_to_nhwc(f1.to(DEV))
    packed = ops.pyramid_build(f2.to(DEV), levels)
    cod = co.to(DEV)
    whole = ops.pyramid_corr_forward(fm1, packed, cod, r, levels, scale=0.25, engine=engine)
    parts = []
    for y0, y1 in bands.band_rows(h, 5, 8):
        parts.append(ops.pyramid_corr_forward(
            fm1[:, y0:y1].contiguous(), packed, cod[:, :, y0:y1].contiguous(), r, levels,
            scale=0.25, engine=engine, map_hw=(h, w)))
    assert torch.equal(torch.cat(parts, dim=3), whole)


def test_band_pyramids_are_slabs_of_the_frame_pyramid():
    b, c, h, w, levels = 2, 64, 270, 96, 4
    f2 = torch.randn(b, c, h, w, generator=torch.Generator().manual_seed(7)).half().to(DEV)
    full = ops.pyramid_build(f2, levels)
    lay = bands.RowBandLayout(b, c, h, w, levels, 8)
    locs = []
    for y0, y1 in lay.bands:
        loc = ops.pyramid_build(f2[:, :, y0:y1].contiguous(), levels)
        pad = loc.new_zeros((b, lay.max_band_elems))
        pad[:, :loc.shape[1]] = loc
        locs.append(pad)
    assert torch.equal(bands.place_band_pyramids(lay, locs), full)


def test_row_band_block_single_process_matches_the_block():
    b, c, h, w, levels, r = 1, 256, 72, 96, 4, 4
    f1, f2, co = _frame(b, c, h, w, torch.float16, seed=9, amp=30.0)
    f1, f2, co = f1.to(DEV), f2.to(DEV), co.to(DEV)
    want = lc.get_localcorr_block(f1, f2, levels, r, corr_mode="localcorr_cuda")(co)
    blk = bands.LocalCorrRowBandBlock(f1, f2, h, num_levels=levels, radius=r)
    got = blk(co)
    assert got.shape == want.shape and torch.equal(got, want)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_rank(rank, world, port, out):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120), device_id=dev)
    try:
        b, c, h, w, levels, r = 1, 128, 99, 80, 4, 4
        f1, f2, co = _frame(b, c, h, w, torch.float16, seed=11, amp=30.0)
        f1, f2, co = f1.to(dev), f2.to(dev), co.to(dev)
        lay = bands.RowBandLayout(b, c, h, w, levels, world)
        y0, y1 = lay.band(rank)
        # whole frame on this rank, for comparison
        x1 = f1.clone().requires_grad_(True)
        x2 = f2.clone().requires_grad_(True)
        whole = lc.get_localcorr_block(x1, x2, levels, r, corr_mode="localcorr_cuda")(co)
        gout = torch.randn(whole.shape, generator=torch.Generator().manual_seed(2)).half()
        gout = gout.to(dev)
        torch.autograd.backward(whole, gout)
        # the band, through the exchange
        b1 = f1[:, :, y0:y1].contiguous().requires_grad_(True)
        b2 = f2[:, :, y0:y1].contiguous().requires_grad_(True)
        blk = bands.LocalCorrRowBandBlock(b1, b2, h, num_levels=levels, radius=r)
        got = blk(co[:, :, y0:y1].contiguous())
        ok_fwd = torch.equal(got, whole[:, :, y0:y1])
        # every rank's loss covers its own rows; the sum over ranks is the
        # whole frame's loss, so each band's fmap grads are the whole frame's rows
        torch.autograd.backward(got, gout[:, :, y0:y1].contiguous())
        ok_g1 = torch.allclose(b1.grad.float(), x1.grad[:, :, y0:y1].float(), rtol=1e-2,
                               atol=1e-2)
        ok_g2 = torch.allclose(b2.grad.float(), x2.grad[:, :, y0:y1].float(), rtol=1e-2,
                               atol=1e-2)
        torch.cuda.synchronize(dev)
        out[rank] = (ok_fwd, ok_g1, ok_g2)
    finally:
        dist.destroy_process_group()


def test_row_bands_on_two_nccl_ranks():
    if torch.cuda.device_count() < 2:
        pytest.skip("two GPUs required")
    import torch.multiprocessing as mp

    world = 2
    port = _free_port()
    with mp.Manager() as mgr:
        out = mgr.dict()
        mp.spawn(_nccl_rank, args=(world, port, out), nprocs=world, join=True)
        res = dict(out)
    for rank in range(world):
        assert res[rank] == (True, True, True), (rank, res[rank])
