"""Row-band split of one frame (localcorr_b200.bands), host side, on CPU.

The band split, the slab bookkeeping, the pyramid exchange (all-gather) and
its backward (reduce-scatter) are checked with gloo ranks on CPU tensors.
Band pyramids are built here by the oracle's pooling chain (test
infrastructure), since the CUDA pyramid build needs a GPU; the GPU tests run
the same exchange on the library's pyramids.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from localcorr_b200 import bands, ops
from oracle import oracle


def _pack(levels):
    """Packed NHWC pyramid [B, sum C*h*w] of a list of NCHW levels (the
    layout of ops.pyramid_build)."""
    b = levels[0].shape[0]
    return torch.cat([p.permute(0, 2, 3, 1).reshape(b, -1) for p in levels], 1).contiguous()


def _band_pyramid(fmap2, y0, y1, levels):
    return _pack(oracle.build_pyramid(fmap2[:, :, y0:y1], levels))


@pytest.mark.parametrize("align", [1, 2, 4, 8])
def test_band_rows_cover_the_frame(align):
    for height in list(range(0, 70)) + [135, 270, 271]:
        for parts in range(1, 10):
            bnd = bands.band_rows(height, parts, align)
            assert len(bnd) == parts
            assert bnd[0][0] == 0 and bnd[-1][1] == height
            for (a0, a1), (b0, b1) in zip(bnd, bnd[1:]):
                assert a1 == b0
            sizes = [y1 - y0 for y0, y1 in bnd]
            assert min(sizes) >= 0
            for y0, y1 in bnd:
                if y1 > y0:
                    assert y0 % align == 0
                    if height >= align:
                        assert y1 - y0 >= align
            whole = [s // align for s in sizes]
            assert max(whole) - min(whole) <= 1 or height < align * parts


def test_band_rows_balance_4k_frame():
    # 270 rows at 8-row alignment over 8 GPUs: 33 units -> 5 + 7 x 4, tail to the last
    assert bands.band_rows(270, 8, 8) == [(0, 40), (40, 72), (72, 104), (104, 136),
                                          (136, 168), (168, 200), (200, 232), (232, 270)]


@pytest.mark.parametrize("shape", [(1, 8, 270, 48, 4, 8), (2, 4, 135, 40, 4, 3),
                                   (1, 4, 20, 16, 4, 4), (1, 4, 33, 20, 2, 5),
                                   (2, 4, 64, 64, 3, 1)])
def test_layout_slabs_tile_the_frame_pyramid(shape):
    b, c, h, w, levels, parts = shape
    lay = bands.RowBandLayout(b, c, h, w, levels, parts)
    lay.check()
    torch.manual_seed(0)
    f2 = torch.randn(b, c, h, w, dtype=torch.float64)
    full = _pack(oracle.build_pyramid(f2, levels))
    locs = []
    for k, (y0, y1) in enumerate(lay.bands):
        loc = _band_pyramid(f2, y0, y1, levels) if y1 > y0 else f2.new_zeros((b, 0))
        assert loc.shape[1] == lay.band_elems[k]
        pad = f2.new_zeros((b, lay.max_band_elems))
        pad[:, :loc.shape[1]] = loc
        locs.append(pad)
    placed = bands.place_band_pyramids(lay, locs)
    # pooling never crosses a band edge: the band pyramids are exact slabs
    assert torch.equal(placed, full)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, shape, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        b, c, h, w, levels = shape
        lay = bands.RowBandLayout(b, c, h, w, levels, world)
        torch.manual_seed(5)  # the same frame on every rank
        f2 = torch.randn(b, c, h, w, dtype=torch.float64)
        y0, y1 = lay.band(rank)
        loc = _band_pyramid(f2, y0, y1, levels) if y1 > y0 else f2.new_zeros((b, 0))
        # forward: every rank ends with the frame's pyramid
        full = bands.gather_pyramid(lay, loc, rank)
        ok_fwd = torch.equal(full, _pack(oracle.build_pyramid(f2, levels)))
        # backward: rank-specific frame gradients, summed back onto the band
        gens = [torch.Generator().manual_seed(100 + r) for r in range(world)]
        grads = [torch.randn(b, lay.frame_elems, generator=g, dtype=torch.float64)
                 for g in gens]
        mine = bands.scatter_pyramid_grad(lay, grads[rank].clone(), rank)
        total = sum(grads)
        want = torch.cat([total[:, fo:fo + n] for (_, fo, n) in lay.slabs[rank]], 1) \
            if lay.slabs[rank] else total.new_zeros((b, 0))
        ok_bwd = torch.allclose(mine, want, rtol=0, atol=1e-12)
        # autograd: GatherPyramid's backward is the reduce-scatter
        leaf = loc.clone().requires_grad_(True)
        fullg = bands.GatherPyramid.apply(leaf, lay, rank, None)
        (fullg * grads[rank]).sum().backward()
        ok_ag = torch.allclose(leaf.grad, want, rtol=0, atol=1e-12)
        out[rank] = (ok_fwd, ok_bwd, ok_ag)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,shape", [(2, (1, 4, 40, 24, 4)), (3, (2, 4, 35, 16, 3)),
                                         (4, (1, 4, 20, 16, 4))])
def test_gloo_ranks_exchange_band_pyramids(world, shape):
    port = _free_port()
    with mp.Manager() as mgr:
        out = mgr.dict()
        mp.spawn(_rank_main, args=(world, port, shape, out), nprocs=world, join=True)
        res = dict(out)
    for rank in range(world):
        assert res[rank] == (True, True, True), (rank, res[rank])


def test_single_band_needs_no_process_group():
    lay = bands.RowBandLayout(1, 4, 16, 16, 2, 1)
    loc = torch.randn(1, lay.frame_elems)
    assert bands.gather_pyramid(lay, loc, 0) is not None
    assert torch.equal(bands.gather_pyramid(lay, loc, 0), loc)
    assert torch.equal(bands.scatter_pyramid_grad(lay, loc, 0), loc)


def test_row_band_block_rejects_host_tensors():
    f = torch.zeros(1, 4, 8, 8)
    with pytest.raises(RuntimeError):
        bands.LocalCorrRowBandBlock(f, f, 8, num_levels=2, radius=1)
    with pytest.raises(ValueError):
        bands.LocalCorrRowBandBlock(f, torch.zeros(1, 4, 16, 8), 16)


def test_map_dims_size_check():
    # fmap2_packed must be the pyramid of the stated map size
    fm1 = torch.zeros(1, 8, 16, 4)
    packed = torch.zeros(1, ops.packed_row_elems(4, 32, 16, 2))
    assert ops._map_dims(fm1, packed, 2, (32, 16)) == (32, 16)
    assert ops._map_dims(fm1, packed, 2, (8, 16)) is None
    with pytest.raises(RuntimeError):
        ops._map_dims(fm1, packed, 2, (30, 16))


def test_bench_row_band_inputs_split_one_frame():
    import bench

    cfg = dict(bench.CONFIGS["raft_4k_rowband"])
    cfg.update(H=40, W=32, C=8, iters=2)
    whole = dict(cfg, band=(0, 40))
    host_w, _ = bench.make_inputs(whole, 0, "cpu")
    parts = []
    for rank, band in enumerate(bands.band_rows(40, 3, 8)):
        host, _ = bench.make_inputs(dict(cfg, band=band), rank, "cpu")
        parts.append(host)
    for key in ("f1", "f2"):
        assert torch.equal(torch.cat([p[key] for p in parts], 2), host_w[key])
    for i in range(cfg["iters"]):
        assert torch.equal(torch.cat([p["coords"][i] for p in parts], 2), host_w["coords"][i])
    cfg["band_rows"] = 8
    assert bench.algorithmic_bytes(cfg, "pyramid_fwd") < bench.algorithmic_bytes(
        dict(cfg, band_rows=40), "pyramid_fwd")
