"""The engine as PyTorch custom operators (``torch.ops.localcorr.*``).

Each operator wraps one C ABI entry point of liblocalcorr_b200.so (through
:mod:`localcorr_b200.ops`), declares its output shapes for fake tensors (so
``torch.compile`` and export trace through it without running it) and carries
its autograd formula, so a call is one opaque node of the graph instead of a
graph break. The reference exposes its CUDA path as a ctypes
``torch.autograd.Function`` (blocks.py:414-537); these operators are that
path's registered form.

Operators (CUDA tensors only; all outputs are new tensors):

* ``nchw_to_nhwc(x)`` / ``nhwc_to_nchw(x)``: [B, C, H, W] <-> [B, H, W, C].
* ``pyramid_build(fmap2, levels)``: the batch-major packed NHWC pyramid
  (2x2 average pooling per level), as ``LocalCorrCudaPyramidBlock`` builds it
  (blocks.py:369-383). Backward: ``pyramid_build_backward``.
* ``pyramid_corr(fmap1, fmap2_packed, coords, radius, levels, dilation,
  ymajor, scale, map_h, map_w)``: ``scale`` x the pyramid local correlation,
  [B, L, (2r+1)^2, H, W]; ``map_h``/``map_w`` > 0 give the level-0 size of the
  map behind ``fmap2_packed`` when it differs from fmap1's grid (row bands),
  0 means fmap1's. Backward: ``pyramid_corr_backward`` (fmap1 gradient in
  the map dtype, packed fmap2 gradient in float32); coords get zeros
  (blocks.py:534-537).
* ``spatial_corr(in1, in2, radius, dilation, scale)``: [B, RD, RD, H, W] on
  NCHW inputs (radius <= 4). Backward: ``spatial_corr_backward``.
"""

from __future__ import annotations

import torch
from torch import Tensor
from torch.library import custom_op

from . import ops

_NS = "localcorr"


def _map_hw(map_h: int, map_w: int):
    return (map_h, map_w) if map_h > 0 and map_w > 0 else None


# ---------------------------------------------------------------------------
# layout
# ---------------------------------------------------------------------------

@custom_op(f"{_NS}::nchw_to_nhwc", mutates_args=(), device_types="cuda")
def nchw_to_nhwc(x: Tensor) -> Tensor:
    return ops.nchw_to_nhwc(x)


@nchw_to_nhwc.register_fake
def _(x):
    b, c, h, w = x.shape
    return x.new_empty((b, h, w, c))


@custom_op(f"{_NS}::nhwc_to_nchw", mutates_args=(), device_types="cuda")
def nhwc_to_nchw(x: Tensor) -> Tensor:
    return ops.nhwc_to_nchw(x)


@nhwc_to_nchw.register_fake
def _(x):
    b, h, w, c = x.shape
    return x.new_empty((b, c, h, w))


def _t_setup(ctx, inputs, output):
    pass


nchw_to_nhwc.register_autograd(lambda ctx, g: torch.ops.localcorr.nhwc_to_nchw(g.contiguous()),
                               setup_context=_t_setup)
nhwc_to_nchw.register_autograd(lambda ctx, g: torch.ops.localcorr.nchw_to_nhwc(g.contiguous()),
                               setup_context=_t_setup)


# ---------------------------------------------------------------------------
# pyramid build
# ---------------------------------------------------------------------------

@custom_op(f"{_NS}::pyramid_build", mutates_args=(), device_types="cuda")
def pyramid_build(fmap2: Tensor, levels: int) -> Tensor:
    return ops.pyramid_build(fmap2, levels)


@pyramid_build.register_fake
def _(fmap2, levels):
    b, c, h, w = fmap2.shape
    return fmap2.new_empty((b, ops.packed_row_elems(c, h, w, levels)))


@custom_op(f"{_NS}::pyramid_build_backward", mutates_args=(), device_types="cuda")
def pyramid_build_backward(grad_packed: Tensor, batch: int, channels: int, height: int,
                           width: int, levels: int, dtype: torch.dtype) -> Tensor:
    return ops.pyramid_build_backward(grad_packed, (batch, channels, height, width), levels,
                                      dtype)


@pyramid_build_backward.register_fake
def _(grad_packed, batch, channels, height, width, levels, dtype):
    return grad_packed.new_empty((batch, channels, height, width), dtype=dtype)


def _pb_setup(ctx, inputs, output):
    fmap2, levels = inputs
    ctx.shape = tuple(fmap2.shape)
    ctx.levels = int(levels)
    ctx.dtype = fmap2.dtype


def _pb_backward(ctx, g):
    b, c, h, w = ctx.shape
    return torch.ops.localcorr.pyramid_build_backward(g.contiguous(), b, c, h, w, ctx.levels,
                                                      ctx.dtype), None


pyramid_build.register_autograd(_pb_backward, setup_context=_pb_setup)


# ---------------------------------------------------------------------------
# pyramid correlation
# ---------------------------------------------------------------------------

@custom_op(f"{_NS}::pyramid_corr", mutates_args=(), device_types="cuda")
def pyramid_corr(fmap1: Tensor, fmap2_packed: Tensor, coords: Tensor, radius: int, levels: int,
                 dilation: int, ymajor: bool, scale: float, map_h: int, map_w: int) -> Tensor:
    return ops.pyramid_corr_forward(fmap1.contiguous(), fmap2_packed.contiguous(),
                                    coords.contiguous(), radius, levels, dilation, ymajor,
                                    scale, map_hw=_map_hw(map_h, map_w))


@pyramid_corr.register_fake
def _(fmap1, fmap2_packed, coords, radius, levels, dilation, ymajor, scale, map_h, map_w):
    b, h, w, _ = fmap1.shape
    rd = 2 * radius + 1
    return fmap1.new_empty((b, levels, rd * rd, h, w))


@custom_op(f"{_NS}::pyramid_corr_backward", mutates_args=(), device_types="cuda")
def pyramid_corr_backward(fmap1: Tensor, fmap2_packed: Tensor, coords: Tensor,
                          corr_grad: Tensor, radius: int, levels: int, dilation: int,
                          ymajor: bool, scale: float, map_h: int,
                          map_w: int) -> tuple[Tensor, Tensor]:
    g1, g2 = ops.pyramid_corr_backward(fmap1.contiguous(), fmap2_packed.contiguous(),
                                       coords.contiguous(), corr_grad.contiguous(), radius,
                                       levels, dilation, ymajor, scale,
                                       map_hw=_map_hw(map_h, map_w))
    return g1, g2


@pyramid_corr_backward.register_fake
def _(fmap1, fmap2_packed, coords, corr_grad, radius, levels, dilation, ymajor, scale, map_h,
      map_w):
    return (torch.empty_like(fmap1, memory_format=torch.contiguous_format),
            fmap2_packed.new_empty(fmap2_packed.shape, dtype=torch.float32))


def _pc_setup(ctx, inputs, output):
    fmap1, fmap2_packed, coords, radius, levels, dilation, ymajor, scale, map_h, map_w = inputs
    ctx.save_for_backward(fmap1, fmap2_packed, coords)
    ctx.params = (radius, levels, dilation, ymajor, scale, map_h, map_w)


def _pc_backward(ctx, corr_grad):
    fmap1, fmap2_packed, coords = ctx.saved_tensors
    g1 = g2 = gc = None
    if ctx.needs_input_grad[0] or ctx.needs_input_grad[1]:
        g1, g2 = torch.ops.localcorr.pyramid_corr_backward(fmap1, fmap2_packed, coords,
                                                           corr_grad.to(fmap1.dtype),
                                                           *ctx.params)
        g2 = g2.to(fmap2_packed.dtype)
    if ctx.needs_input_grad[2]:
        # RAFT detaches the sampling coordinates: zeros, as the reference
        # returns (blocks.py:534-537).
        gc = torch.zeros_like(coords)
    return g1, g2, gc, None, None, None, None, None, None, None


pyramid_corr.register_autograd(_pc_backward, setup_context=_pc_setup)


# ---------------------------------------------------------------------------
# spatial correlation
# ---------------------------------------------------------------------------

@custom_op(f"{_NS}::spatial_corr", mutates_args=(), device_types="cuda")
def spatial_corr(in1: Tensor, in2: Tensor, radius: int, dilation: int, scale: float) -> Tensor:
    return ops.spatial_forward(in1.contiguous(), in2.contiguous(), radius, dilation, scale)


@spatial_corr.register_fake
def _(in1, in2, radius, dilation, scale):
    b, c, h, w = in1.shape
    rd = 2 * radius + 1
    return in1.new_empty((b, rd, rd, h, w))


@custom_op(f"{_NS}::spatial_corr_backward", mutates_args=(), device_types="cuda")
def spatial_corr_backward(in1: Tensor, in2: Tensor, grad_out: Tensor, radius: int,
                          dilation: int, scale: float) -> tuple[Tensor, Tensor]:
    g1, g2 = ops.spatial_backward(in1.contiguous(), in2.contiguous(), grad_out.contiguous(),
                                  radius, dilation, scale)
    return g1, g2


@spatial_corr_backward.register_fake
def _(in1, in2, grad_out, radius, dilation, scale):
    return (torch.empty_like(in1, memory_format=torch.contiguous_format),
            torch.empty_like(in2, memory_format=torch.contiguous_format))


def _sc_setup(ctx, inputs, output):
    in1, in2, radius, dilation, scale = inputs
    ctx.save_for_backward(in1, in2)
    ctx.params = (radius, dilation, scale)


def _sc_backward(ctx, g):
    in1, in2 = ctx.saved_tensors
    g1, g2 = torch.ops.localcorr.spatial_corr_backward(in1, in2, g.to(in1.dtype), *ctx.params)
    return (g1 if ctx.needs_input_grad[0] else None,
            g2 if ctx.needs_input_grad[1] else None, None, None, None)


spatial_corr.register_autograd(_sc_backward, setup_context=_sc_setup)
