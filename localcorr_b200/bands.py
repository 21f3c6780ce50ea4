"""Row bands: one large frame's pyramid correlation split over the GPUs of a node.

The reference runs one frame on one device (blocks.py:337-411). For a frame
too large for one GPU's time budget (a 4K frame at batch 1), the pixel rows
are split into bands, one per rank (one process per GPU):

* fmap1, coords and the correlation output are split by rows; every rank
  computes exactly its rows of the whole-frame output.
* Each rank also holds its rows of fmap2 and builds the pyramid levels of its
  band (bands start on multiples of 2^(levels-1) rows, so 2x2 pooling never
  crosses a band edge and a band's level-l rows are rows
  [y0 >> l, y1 >> l) of the whole frame's level l).
* One exchange step per frame: the band pyramids are all-gathered into the
  whole frame's packed pyramid on every rank (NCCL over NVLink). The lookups
  of the frame then run locally through the map-size-decoupled entry points
  (``launchLocalCorrB200PyramidForwardMapDims``): fmap1/coords of the band,
  pyramid of the frame, coordinates in whole-frame pixels.
* Backward (training on bands): each rank's lookups produce a gradient of
  the whole-frame pyramid; a reduce-scatter returns to each rank the sum over
  ranks of its own band's slabs, which the band's pyramid backward folds into
  its fmap2 rows.

The exchange moves every level of every band (the whole packed pyramid,
88 MB in float16 for a 270x480x256 frame) rather than only the rows a band's
coordinates reach: it is one collective per frame, amortised over the
frame's lookups, and needs no data-dependent sizes.
"""

from __future__ import annotations

import math

import torch
import torch.distributed as dist

from . import ops

__all__ = [
    "band_rows",
    "RowBandLayout",
    "gather_pyramid",
    "place_band_pyramids",
    "scatter_pyramid_grad",
    "GatherPyramid",
    "LocalCorrRowBandBlock",
]


def band_rows(height: int, parts: int, align: int) -> list[tuple[int, int]]:
    """Split rows [0, height) into ``parts`` bands [y0, y1).

    Band starts are multiples of ``align``; the whole ``align``-row units are
    dealt out as evenly as possible, the larger shares first, and the rows
    past the last whole unit join the last band that holds a unit, so every
    non-empty band holds at least ``align`` rows (when the frame does). With
    more parts than units, some bands are empty (y0 == y1)."""
    if parts < 1 or align < 1 or height < 0:
        raise ValueError("band_rows needs parts >= 1, align >= 1, height >= 0")
    units = height // align
    bu = [(units * k + parts - 1) // parts for k in range(parts + 1)]
    out = [(align * bu[k], align * bu[k + 1]) for k in range(parts)]
    live = [k for k in range(parts) if bu[k + 1] > bu[k]]
    last = live[-1] if live else 0
    out[last] = (out[last][0], height)
    for k in range(last + 1, parts):
        out[k] = (height, height)
    return out


class RowBandLayout:
    """Where each band's pyramid slabs sit in its own and in the frame's packed
    pyramid (batch-major, levels concatenated, NHWC per level: the layout of
    ``ops.pyramid_build``)."""

    def __init__(self, batch: int, channels: int, height: int, width: int, levels: int,
                 parts: int):
        self.B, self.C, self.H, self.W, self.L = batch, channels, height, width, levels
        self.parts = parts
        self.align = 1 << (levels - 1)
        self.bands = band_rows(height, parts, self.align)
        self.frame_elems = ops.packed_row_elems(channels, height, width, levels)
        # per band: its own packed row length and, per level, (band offset,
        # frame offset, elements) of its slab in one batch row
        self.band_elems = []
        self.slabs = []
        frame_off = 0
        frame_level_off = []
        for l in range(levels):
            frame_level_off.append(frame_off)
            frame_off += channels * (height >> l) * (width >> l)
        for (y0, y1) in self.bands:
            hb = y1 - y0
            slabs = []
            off = 0
            if hb > 0:
                for l in range(levels):
                    # y0 is a multiple of 2^l, so this is also (y1 - y0) >> l,
                    # the band pyramid's level-l row count
                    rows = (y1 >> l) - (y0 >> l)
                    n = rows * (width >> l) * channels
                    fo = frame_level_off[l] + (y0 >> l) * (width >> l) * channels
                    slabs.append((off, fo, n))
                    off += n
            self.band_elems.append(off)
            self.slabs.append(slabs)
        self.max_band_elems = max(self.band_elems) if self.band_elems else 0

    def band(self, rank: int) -> tuple[int, int]:
        return self.bands[rank]

    def check(self) -> None:
        """Every frame position is covered by exactly one band slab."""
        for b_slabs, (y0, y1), n in zip(self.slabs, self.bands, self.band_elems):
            if y1 > y0 and n != ops.packed_row_elems(self.C, y1 - y0, self.W, self.L):
                raise AssertionError("band slab sizes disagree with the band pyramid")
        covered = sum(n for slabs in self.slabs for (_, _, n) in slabs)
        if covered != self.frame_elems:
            raise AssertionError("band slabs do not tile the frame pyramid")


def _pack_send(layout: RowBandLayout, local: torch.Tensor, rank: int) -> torch.Tensor:
    n = layout.band_elems[rank]
    send = local.new_zeros((layout.B, layout.max_band_elems))
    if n:
        send[:, :n].copy_(local.reshape(layout.B, n))
    return send


def place_band_pyramids(layout: RowBandLayout, bands: list[torch.Tensor]) -> torch.Tensor:
    """Frame pyramid [B, frame_elems] from every band's pyramid (bands[k]:
    [B, >= band_elems[k]], band k's packed pyramid first)."""
    full = bands[0].new_empty((layout.B, layout.frame_elems))
    for k, slabs in enumerate(layout.slabs):
        for (bo, fo, n) in slabs:
            full[:, fo:fo + n].copy_(bands[k][:, bo:bo + n])
    return full


def gather_pyramid(layout: RowBandLayout, local: torch.Tensor, rank: int,
                   group=None) -> torch.Tensor:
    """All-gather the band pyramids into the frame's packed pyramid.

    local: this rank's band pyramid [B, band_elems[rank]] (``ops.pyramid_build``
    of its fmap2 rows). Returns [B, frame_elems] on every rank. One all-gather
    of equal-size (padded) buffers, then each band's slabs are placed."""
    if layout.parts == 1:
        return local.reshape(layout.B, layout.frame_elems)
    send = _pack_send(layout, local, rank)
    recv = [torch.empty_like(send) for _ in range(layout.parts)]
    dist.all_gather(recv, send, group=group)
    return place_band_pyramids(layout, recv)


def scatter_pyramid_grad(layout: RowBandLayout, grad_full: torch.Tensor, rank: int,
                         group=None) -> torch.Tensor:
    """Reduce-scatter of the frame pyramid's gradient back to the bands.

    grad_full: this rank's gradient of the frame pyramid [B, frame_elems].
    Returns [B, band_elems[rank]]: the sum over ranks of this band's slabs."""
    parts = layout.parts
    if parts == 1:
        return grad_full
    send = grad_full.new_zeros((parts, layout.B, layout.max_band_elems))
    for k, slabs in enumerate(layout.slabs):
        for (bo, fo, n) in slabs:
            send[k, :, bo:bo + n].copy_(grad_full[:, fo:fo + n])
    out = grad_full.new_empty((layout.B, layout.max_band_elems))
    # flat views: input = world_size consecutive outputs (NCCL and gloo)
    dist.reduce_scatter_tensor(out.view(-1), send.view(-1), group=group)
    return out[:, :layout.band_elems[rank]].contiguous()


class GatherPyramid(torch.autograd.Function):
    """gather_pyramid with the reduce-scatter as its backward."""

    @staticmethod
    def forward(ctx, local, layout, rank, group):
        ctx.layout, ctx.rank, ctx.group = layout, rank, group
        return gather_pyramid(layout, local, rank, group)

    @staticmethod
    def backward(ctx, g):
        # half-precision gradients are summed over ranks in float32; autograd
        # casts the result to the band's dtype
        g = g.contiguous()
        if g.dtype in (torch.float16, torch.bfloat16):
            g = g.float()
        return scatter_pyramid_grad(ctx.layout, g, ctx.rank, ctx.group), None, None, None


class LocalCorrRowBandBlock:
    """The RAFT correlation block (``LocalCorrCudaPyramidBlock``,
    blocks.py:337-411) for one row band of a frame split over the ranks of a
    process group.

    fmap1_band, fmap2_band: rows [y0, y1) of the frame's [B, C, H, W] maps,
    where (y0, y1) = ``RowBandLayout.band(rank)``; ``height`` is the frame's H.
    ``block(coords_band)`` with coords_band [B, 2, y1 - y0, W] in whole-frame
    level-0 pixels returns rows [y0, y1) of the whole-frame block output
    [B, L*(2r+1)^2, y1 - y0, W], scaled by 1/sqrt(C). Construction is the
    frame's one exchange step (collective: every rank of the group constructs
    its block together)."""

    def __init__(self, fmap1_band: torch.Tensor, fmap2_band: torch.Tensor, height: int,
                 num_levels: int = 4, radius: int = 4, group=None):
        if fmap1_band.dim() != 4 or fmap2_band.shape != fmap1_band.shape:
            raise ValueError("fmap1_band and fmap2_band must be [B, C, rows, W] of one shape")
        if not (fmap1_band.is_cuda and fmap2_band.is_cuda):
            raise RuntimeError("localcorr_b200 requires the feature maps on a CUDA device")
        if fmap1_band.dtype not in (torch.float32, torch.float16) or \
                fmap2_band.dtype != fmap1_band.dtype:
            raise RuntimeError("localcorr_b200 requires float32 or float16 feature maps of one "
                               f"dtype, but got {fmap1_band.dtype} and {fmap2_band.dtype}.")
        self.num_levels = int(num_levels)
        self.radius = int(radius)
        self.group = group
        single = not (dist.is_available() and dist.is_initialized())
        self.rank = 0 if single else dist.get_rank(group)
        parts = 1 if single else dist.get_world_size(group)
        b, c, hb, w = fmap1_band.shape
        self.dim = c
        self.height, self.width = int(height), w
        self.layout = RowBandLayout(b, c, self.height, w, self.num_levels, parts)
        y0, y1 = self.layout.band(self.rank)
        if hb != y1 - y0:
            raise ValueError(f"rank {self.rank} holds rows [{y0}, {y1}) of a {height}-row "
                             f"frame but got {hb} rows")
        self.rows = (y0, y1)
        self.scale = 1.0 / math.sqrt(c)
        if hb > 0:
            self.fmap1 = torch.ops.localcorr.nchw_to_nhwc(fmap1_band)
            local = torch.ops.localcorr.pyramid_build(fmap2_band, self.num_levels)
        else:
            self.fmap1 = fmap1_band.new_empty((b, 0, w, c))
            local = fmap2_band.new_empty((b, 0))
        if parts == 1:
            self.fmap2_packed = local
        else:
            self.fmap2_packed = GatherPyramid.apply(local, self.layout, self.rank, group)

    def __call__(self, coords_band: torch.Tensor) -> torch.Tensor:
        b, _, hb, w = coords_band.shape
        rd = 2 * self.radius + 1
        if not coords_band.is_cuda:
            raise RuntimeError("localcorr_b200 requires coords on a CUDA device")
        if coords_band.dtype not in (torch.float32, torch.float16):
            raise RuntimeError(f"coords must be float32 or float16, got {coords_band.dtype}")
        if hb != self.rows[1] - self.rows[0]:
            raise ValueError(f"coords cover {hb} rows, the band has "
                             f"{self.rows[1] - self.rows[0]}")
        if hb == 0:
            return coords_band.new_empty((b, self.num_levels * rd * rd, 0, w),
                                         dtype=self.fmap1.dtype)
        corr = torch.ops.localcorr.pyramid_corr(self.fmap1, self.fmap2_packed, coords_band,
                                                self.radius, self.num_levels, 1, False,
                                                self.scale, self.height, self.width)
        return corr.reshape(b, -1, hb, w)
