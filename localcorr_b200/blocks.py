"""RAFT-style local correlation blocks and PWC-style samplers (public API).

Mirrors the reference module blocks.py: the same factory signatures
(get_localcorr_block, blocks.py:1182-1245; get_localcorr_sampler,
blocks.py:785-835), class names, attributes, output layouts and errors.
Every accepted corr_mode runs the single sm_100a engine of
liblocalcorr_b200.so; there is no Triton path, no device auto-dispatch and no
CPU fallback, so CPU tensors raise RuntimeError at call time as the
reference's CUDA mode does (blocks.py:552-557).

Layouts:
  block(coords) -> [B, num_levels*(2r+1)^2, H, W], scaled by 1/sqrt(C),
                   channel d = iy + (2r+1)*ix per level (RAFT order);
  sampler(in1, in2) -> [B, P, P, H, W], unscaled, [b, dy_idx, dx_idx, h, w].
"""

from __future__ import annotations

import math

import torch

from . import _lib
from . import ops
from .backend import use_onnx_generic_ops

__all__ = [
    "get_cuda_pyramid_library",
    "get_localcorr_block",
    "get_localcorr_sampler",
    "LocalCorrCudaPyramidBlock",
    "LocalCorrCudaPyramidFunction",
    "LocalCorrCudaPyramidOnnx",
    "LocalCorrCudaPyramidSpatialBlock",
    "LocalCorrCudaPyramidSpatialOnnx",
    "LocalCorrCudaSpatialSampler",
    "LocalCorrOnnxBlock",
    "LocalCorrOnnxSpatialSampler",
    "LocalCorrSyclBlock",
    "LocalCorrSyclSpatialSampler",
    "LocalCorrTritonBlock",
    "LocalCorrTritonFusedBlock",
]

_CORR_MODES = ("localcorr_triton", "localcorr_cuda", "localcorr_onnx", "localcorr_sycl",
               "localcorr_auto")


def get_cuda_pyramid_library():
    """Return the ctypes handle of liblocalcorr_b200.so, or None if not built.

    Counterpart of the reference get_cuda_pyramid_library (blocks.py:74-131):
    the handle exposes launchLocalCorrCudaPyramidForward/Backward with the
    reference's argtypes, plus this library's extended entry points.
    """
    return _lib.load_library()


class LocalCorrCudaPyramidOnnx(torch.autograd.Function):
    """ONNX-export wrapper of the fused pyramid correlation (blocks.py:156-204).

    forward() only materialises the output shape; symbolic() records one
    custom_ops::LocalCorrCudaPyramid node (attributes radius/levels/dilation/
    ymajor) that the TensorRT plugin built against this library computes.
    """

    @staticmethod
    def forward(ctx, fmap1, fmap2_packed, coords, radius, num_levels, dilation=1):
        radius = int(radius)
        num_levels = int(num_levels)
        b, h, w, _ = fmap1.shape
        rd = 2 * radius + 1
        return fmap1.new_empty((b, num_levels, rd * rd, h, w))

    @staticmethod
    def symbolic(g, fmap1, fmap2_packed, coords, radius, num_levels, dilation=1):
        node = g.op("custom_ops::LocalCorrCudaPyramid", fmap1, fmap2_packed, coords,
                    radius_i=int(radius), levels_i=int(num_levels), dilation_i=int(dilation),
                    ymajor_i=0)
        f1s = fmap1.type().sizes()
        cs = coords.type().sizes()
        if f1s is not None and cs is not None:
            rd = 2 * int(radius) + 1
            node.setType(fmap1.type().with_sizes([cs[0], int(num_levels), rd * rd, f1s[1], f1s[2]]))
        return node


class LocalCorrCudaPyramidSpatialOnnx(torch.autograd.Function):
    """ONNX-export wrapper of the single-level dilated spatial correlation
    (blocks.py:951-1043): forward() materialises [B, rd*rd, H, W]."""

    @staticmethod
    def forward(ctx, fmap1, fmap2, coords, radius, dilation, normalize):
        radius = int(radius)
        b, h, w, _ = fmap1.shape
        rd = 2 * radius + 1
        return fmap1.new_empty((b, rd * rd, h, w))

    @staticmethod
    def symbolic(g, fmap1, fmap2, coords, radius, dilation, normalize):
        f1s = fmap1.type().sizes() if fmap1.type() is not None else None
        f2s = fmap2.type().sizes() if fmap2.type() is not None else None
        if f2s is not None:
            bsz = f2s[0]
        elif f1s is not None:
            bsz = f1s[0]
        else:
            raise RuntimeError(
                "spatial plugin-node export packs fmap2 per image and so needs a static "
                "batch dimension on fmap1 or fmap2; the traced graph has no shape for either")
        packed = g.op("Reshape", fmap2,
                      g.op("Constant", value_t=torch.tensor([bsz, -1], dtype=torch.int64)))
        node = g.op("custom_ops::LocalCorrCudaPyramid", fmap1, packed, coords,
                    radius_i=int(radius), levels_i=1, dilation_i=int(dilation), ymajor_i=1)
        cs = coords.type().sizes() if coords.type() is not None else None
        if f1s is not None and cs is not None:
            rd = 2 * int(radius) + 1
            node.setType(fmap1.type().with_sizes([cs[0], 1, rd * rd, f1s[1], f1s[2]]))
            node = g.op("Reshape", node, g.op(
                "Constant",
                value_t=torch.tensor([cs[0], rd * rd, f1s[1], f1s[2]], dtype=torch.int64)))
        return node


class LocalCorrCudaPyramidFunction(torch.autograd.Function):
    """Autograd Function over the reference-compatible C ABI
    (launchLocalCorrCudaPyramidForward/Backward), same signature and contract
    as the reference Function (blocks.py:414-537): fmap1 NHWC, fmap2_packed
    batch-major, coords planar x/y of the same dtype; output unscaled
    [B, L, RD^2, H, W]; grads for fmap1 and fmap2_packed, zeros for coords.
    """

    @staticmethod
    def forward(ctx, fmap1, fmap2_packed, coords, radius, num_levels, dilation, ymajor):
        lib = _lib.require_library()
        coords = coords.contiguous()
        fmap1 = fmap1.contiguous()
        fmap2_packed = fmap2_packed.contiguous()
        b, h, w, c = fmap1.shape
        rd = 2 * radius + 1
        corr = fmap1.new_empty((b, num_levels, rd * rd, h, w))
        stream = torch.cuda.current_stream(fmap1.device).cuda_stream
        with torch.cuda.device(fmap1.device):
            ok = lib.launchLocalCorrCudaPyramidForward(
                fmap1.data_ptr(), fmap2_packed.data_ptr(), coords.data_ptr(), corr.data_ptr(),
                b, h, w, c, radius, num_levels, dilation, fmap1.dtype == torch.float16, ymajor,
                stream)
        if not ok:
            raise RuntimeError(
                "localcorr CUDA kernel launch failed (e.g. shared-memory overflow for this "
                f"radius/channel count): {_lib.last_error(lib)}")
        ctx.save_for_backward(fmap1, fmap2_packed, coords)
        ctx.kernel_params = (int(radius), int(num_levels), int(dilation), bool(ymajor))
        return corr

    @staticmethod
    def backward(ctx, corr_grad):
        fmap1, fmap2_packed, coords = ctx.saved_tensors
        radius, num_levels, dilation, ymajor = ctx.kernel_params
        lib = _lib.require_library()
        corr_grad = corr_grad.contiguous()
        b, h, w, c = fmap1.shape
        stream = torch.cuda.current_stream(fmap1.device).cuda_stream
        fmap1_grad = torch.empty_like(fmap1)
        f2g32 = torch.zeros(fmap2_packed.shape, dtype=torch.float32, device=fmap2_packed.device)
        with torch.cuda.device(fmap1.device):
            ok = lib.launchLocalCorrCudaPyramidBackward(
                fmap1.data_ptr(), fmap2_packed.data_ptr(), coords.data_ptr(),
                corr_grad.data_ptr(), fmap1_grad.data_ptr(), f2g32.data_ptr(), b, h, w, c,
                radius, num_levels, dilation, fmap1.dtype == torch.float16, ymajor, stream)
        if not ok:
            raise RuntimeError(
                "localcorr CUDA backward kernel launch failed (e.g. shared-memory overflow for "
                f"this channel count): {_lib.last_error(lib)}")
        fmap2_grad = f2g32 if fmap2_packed.dtype == torch.float32 else f2g32.to(fmap2_packed.dtype)
        return fmap1_grad, fmap2_grad, torch.zeros_like(coords), None, None, None, None


def _localcorr_cuda_pyramid_forward(fmap1, fmap2_packed, coords, radius, num_levels,
                                    dilation=1, ymajor=False):
    """Guards + LocalCorrCudaPyramidFunction, as the reference helper
    (blocks.py:540-588): CUDA device, built library, dtype, coords dtype."""
    if not fmap1.is_cuda:
        raise RuntimeError(
            'corr_mode="localcorr_cuda" requires the feature maps to be on a CUDA device, '
            f"but they are on {fmap1.device}.")
    lib = get_cuda_pyramid_library()
    if lib is None:
        raise ImportError(
            'corr_mode="localcorr_cuda" requires the CUDA kernel library, but it has not been '
            "built (or could not be loaded). Build it with: python -m localcorr_b200.csrc.build")
    if fmap1.dtype not in (torch.float32, torch.float16):
        raise RuntimeError(
            'corr_mode="localcorr_cuda" requires float32 or float16 feature maps, but got '
            f"{fmap1.dtype}.")
    if coords.dtype != fmap1.dtype:
        raise RuntimeError(
            'corr_mode="localcorr_cuda" requires the coords dtype to match the feature maps '
            f"dtype, but got {coords.dtype} and {fmap1.dtype}.")
    return LocalCorrCudaPyramidFunction.apply(fmap1, fmap2_packed, coords, int(radius),
                                              int(num_levels), int(dilation), bool(ymajor))


class LocalCorrCudaPyramidBlock:
    """Local correlation with all pyramid levels in one engine call.

    Construction (blocks.py:354-383) prepares, with this library's kernels and
    autograd support, the NHWC fmap1 (``self.fmap1``) and the batch-major
    packed pyramid (``self.fmap2_packed``, views per level in
    ``self.fmap2_pyramid``). Calling the block with coords [B, 2, H, W]
    (x, y; level-0 pixels; float32 or float16) returns the correlation
    scaled by 1/sqrt(C), the scale fused into the kernel.
    """

    onnx_generic = False

    def __init__(self, fmap1, fmap2, num_levels=4, radius=4, onnx_generic: bool = False):
        self.num_levels = int(num_levels)
        self.radius = int(radius)
        self.dim = fmap1.shape[1]
        self.onnx_generic = bool(onnx_generic) or type(self).onnx_generic
        self._on_cuda = bool(fmap1.is_cuda and fmap2.is_cuda)
        if not self._on_cuda or torch.onnx.is_in_onnx_export():
            # Nothing runs on the host: the NCHW maps are kept and the call
            # raises (eager) or records the export node.
            self.fmap1_nchw = fmap1
            self.fmap2_nchw = fmap2
            return
        if fmap1.dtype not in (torch.float32, torch.float16) or fmap2.dtype != fmap1.dtype:
            raise RuntimeError(
                "localcorr_b200 requires float32 or float16 feature maps of one dtype, but got "
                f"{fmap1.dtype} and {fmap2.dtype}.")
        self.fmap1 = torch.ops.localcorr.nchw_to_nhwc(fmap1)
        self.fmap2_packed = torch.ops.localcorr.pyramid_build(fmap2, self.num_levels)
        # Lookups read detached copies of the prepared maps and send their
        # gradients through one token into shared accumulators (see
        # ops.LookupGrads); the attributes above stay differentiable for
        # callers that use them directly.
        self._grads = None
        self._token = None
        # Under torch.compile the lookups stay registered custom operators
        # (torch.ops.localcorr.pyramid_corr, one graph node each, no break);
        # eagerly they share one pair of gradient accumulators.
        if (torch.is_grad_enabled() and (fmap1.requires_grad or fmap2.requires_grad)
                and not torch.compiler.is_compiling()):
            self._grads = ops.LookupGrads(self.fmap1.detach(), self.fmap2_packed.detach(),
                                          fmap2.shape, self.num_levels)
            self._token = ops.LookupGradSink.apply(fmap1, fmap2, self._grads)
        b, c, h, w = fmap2.shape
        self.fmap2_pyramid = []
        off = 0
        for hl, wl in ops.level_shapes(h, w, self.num_levels):
            n = c * hl * wl
            self.fmap2_pyramid.append(self.fmap2_packed[:, off:off + n].view(b, hl, wl, c))
            off += n

    def use_generic_export_ops(self) -> bool:
        return use_onnx_generic_ops() or (self.onnx_generic and torch.onnx.is_in_onnx_export())

    def __call__(self, coords):
        b, _, h, w = coords.shape
        if torch.onnx.is_in_onnx_export():
            return self._export(coords)
        if not self._on_cuda or not coords.is_cuda:
            raise RuntimeError(
                "localcorr_b200 requires the feature maps and coords to be on a CUDA device, "
                f"but they are on {self.fmap1_nchw.device if not self._on_cuda else coords.device}.")
        _lib.require_library()
        if coords.dtype not in (torch.float32, torch.float16):
            raise RuntimeError(f"coords must be float32 or float16, got {coords.dtype}")
        scale = 1.0 / math.sqrt(self.dim)
        if self._token is not None and torch.is_grad_enabled():
            corr = ops.PyramidLookup.apply(self._token, coords, self._grads, self.radius,
                                           self.num_levels, scale)
        else:
            corr = torch.ops.localcorr.pyramid_corr(self.fmap1, self.fmap2_packed, coords,
                                                    self.radius, self.num_levels, 1, False,
                                                    scale, 0, 0)
        return corr.reshape(b, -1, h, w)

    def _export(self, coords):
        if self.use_generic_export_ops():
            raise NotImplementedError(
                "standard-ops ONNX export of the correlation is not provided by localcorr_b200; "
                "export with the plugin node (the default backend)")
        fmap1 = self.fmap1_nchw.permute(0, 2, 3, 1).contiguous()
        pyr = [self.fmap2_nchw]
        for _ in range(1, self.num_levels):
            pyr.append(torch.nn.functional.avg_pool2d(pyr[-1], 2, stride=2))
        packed = torch.cat([p.permute(0, 2, 3, 1).reshape(p.shape[0], -1) for p in pyr], dim=1)
        corr = LocalCorrCudaPyramidOnnx.apply(fmap1, packed, coords, self.radius,
                                              self.num_levels)
        b, _, h, w = coords.shape
        return corr.reshape(b, -1, h, w) / math.sqrt(self.dim)


class LocalCorrTritonFusedBlock(LocalCorrCudaPyramidBlock):
    """corr_mode="localcorr_triton" (reference: fused Triton kernel,
    blocks.py:265-334); here the same sm_100a engine as localcorr_cuda."""


class LocalCorrTritonBlock(LocalCorrCudaPyramidBlock):
    """Per-level reference block of the reference (blocks.py:207-262); here the
    sm_100a engine (all levels in one call)."""


class LocalCorrOnnxBlock(LocalCorrCudaPyramidBlock):
    """corr_mode="localcorr_onnx" (blocks.py:1142-1179): eager = sm_100a engine."""

    onnx_generic = True


class LocalCorrSyclBlock(LocalCorrCudaPyramidBlock):
    """corr_mode="localcorr_sycl" (blocks.py:951-1043 on Intel); on NVIDIA the
    sm_100a engine."""


def get_localcorr_block(fmap1: torch.Tensor, fmap2: torch.Tensor, num_levels: int = 4,
                        radius: int = 4, corr_mode: str = "localcorr_triton",
                        xpu_backend: str = "sycl"):
    """Create a RAFT-style local correlation block (blocks.py:1182-1245).

    All corr modes (localcorr_triton, localcorr_cuda, localcorr_onnx,
    localcorr_sycl, localcorr_auto; case-insensitive) run the sm_100a engine;
    the mode only selects the class (and localcorr_onnx's export flag).
    xpu_backend is accepted for signature compatibility. Unknown modes raise
    ValueError.
    """
    mode = corr_mode.lower()
    cls = {
        "localcorr_triton": LocalCorrTritonFusedBlock,
        "localcorr_cuda": LocalCorrCudaPyramidBlock,
        "localcorr_onnx": LocalCorrOnnxBlock,
        "localcorr_sycl": LocalCorrSyclBlock,
        "localcorr_auto": LocalCorrCudaPyramidBlock,
    }.get(mode)
    if cls is None:
        raise ValueError(f"Unknown local corr_mode: {corr_mode}")
    return cls(fmap1=fmap1, fmap2=fmap2, num_levels=num_levels, radius=radius)


# ---------------------------------------------------------------------------
# PWC-Net style samplers
# ---------------------------------------------------------------------------

class _SpatialSamplerBase:
    """Common logic of the spatial samplers (blocks.py:623-668): the
    kernel_size/stride/padding/dilation asserts and the [B,P,P,H,W] layout."""

    def __init__(self, kernel_size=1, patch_size=9, stride=1, padding=0, dilation=1,
                 dilation_patch=1):
        assert kernel_size == 1, "Only kernel_size=1 is supported."
        assert stride == 1, "Only stride=1 is supported."
        assert padding == 0, "Only padding=0 is supported."
        assert dilation == 1, "Only dilation=1 is supported."
        self.md = patch_size // 2
        self.patch_size = patch_size
        self.dilation_patch = dilation_patch

    def __call__(self, input1, input2):
        b, _, h, w = input1.shape
        if torch.onnx.is_in_onnx_export():
            fmap1 = input1.permute(0, 2, 3, 1).contiguous()
            fmap2 = input2.permute(0, 2, 3, 1).contiguous()
            coords = ops.identity_coords(b, h, w, input1.dtype, input1.device)
            corr = LocalCorrCudaPyramidSpatialOnnx.apply(fmap1, fmap2, coords, self.md,
                                                         self.dilation_patch, None)
            return corr.view(b, self.patch_size, self.patch_size, h, w)
        if not (input1.is_cuda and input2.is_cuda):
            raise RuntimeError(
                "localcorr_b200 spatial correlation requires inputs on a CUDA device, but they "
                f"are on {input1.device}.")
        _lib.require_library()
        if input1.dtype not in (torch.float32, torch.float16):
            raise RuntimeError(
                f"localcorr_b200 requires float32 or float16 inputs, but got {input1.dtype}.")
        out = ops.spatial_corr(input1, input2, self.md, self.dilation_patch, 1.0)
        return out.view(b, self.patch_size, self.patch_size, h, w)


class LocalCorrCudaSpatialSampler(_SpatialSamplerBase):
    """corr_mode="localcorr_cuda", PWC-Net style (blocks.py:671-694), trainable."""


class LocalCorrOnnxSpatialSampler(_SpatialSamplerBase):
    """corr_mode="localcorr_onnx" sampler (blocks.py:738-782); eager = sm_100a engine."""


class LocalCorrSyclSpatialSampler(_SpatialSamplerBase):
    """corr_mode="localcorr_sycl" sampler (blocks.py:697-735); on NVIDIA the
    sm_100a engine."""


class TritonSpatialCorrelationSampler(_SpatialSamplerBase):
    """corr_mode="localcorr_triton" sampler (triton/spatial_corr.py:210-233);
    here the sm_100a engine."""


def get_localcorr_sampler(patch_size: int = 9, dilation_patch: int = 1,
                          corr_mode: str = "localcorr_triton", xpu_backend: str = "sycl"):
    """Create a PWC-Net-style spatial correlation sampler (blocks.py:785-835),
    equivalent to SpatialCorrelationSampler(kernel_size=1, patch_size,
    padding=0, dilation_patch). All modes run the sm_100a engine."""
    mode = corr_mode.lower()
    kwargs = dict(kernel_size=1, patch_size=patch_size, padding=0,
                  dilation_patch=dilation_patch)
    if mode == "localcorr_auto":
        from .spatial_corr import LocalCorrCudaPyramidSampler

        return LocalCorrCudaPyramidSampler(xpu_backend=xpu_backend, **kwargs)
    cls = {
        "localcorr_triton": TritonSpatialCorrelationSampler,
        "localcorr_cuda": LocalCorrCudaSpatialSampler,
        "localcorr_onnx": LocalCorrOnnxSpatialSampler,
        "localcorr_sycl": LocalCorrSyclSpatialSampler,
    }.get(mode)
    if cls is None:
        raise ValueError(f"Unknown local corr_mode: {corr_mode}")
    return cls(**kwargs)


class LocalCorrCudaPyramidSpatialBlock:
    """Single-level dilated spatial correlation, FlowNetC style
    (blocks.py:1046-1139): corr[b, iy*rd+ix, h, w] = sum_c fmap1[b,c,h,w] *
    fmap2[b,c,h+dil*(iy-r), w+dil*(ix-r)], then normalize "sqrt" (/sqrt(C)),
    "dim" (/C) or None. coords passed to __call__ are ignored. The reference
    computes it with shifted torch slices; here the spatial kernel (radius
    <= 4) or the one-level pyramid engine (larger radius)."""

    def __init__(self, fmap1, fmap2, radius=10, dilation=2, normalize="sqrt"):
        self.radius = radius
        self.dilation = dilation
        self.dim = fmap1.shape[1]
        self.fmap1 = fmap1
        self.fmap2 = fmap2
        self.normalize = normalize
        self._coords = None

    def _scale(self) -> float:
        if self.normalize == "sqrt":
            return 1.0 / math.sqrt(self.dim)
        if self.normalize == "dim":
            return 1.0 / self.dim
        return 1.0

    def _identity_coords(self, b, h, w, dtype, device):
        if (self._coords is None or self._coords.shape[0] != b or self._coords.shape[2] != h
                or self._coords.shape[3] != w or self._coords.dtype != dtype
                or self._coords.device != device):
            self._coords = ops.identity_coords(b, h, w, dtype, device)
        return self._coords

    def __call__(self, coords=None):
        b, c, h, w = self.fmap1.shape
        rd = 2 * self.radius + 1
        if torch.onnx.is_in_onnx_export():
            f1 = self.fmap1.permute(0, 2, 3, 1).contiguous()
            f2 = self.fmap2.permute(0, 2, 3, 1).contiguous()
            grid = self._identity_coords(b, h, w, self.fmap1.dtype, self.fmap1.device)
            corr = LocalCorrCudaPyramidSpatialOnnx.apply(f1, f2, grid, self.radius,
                                                         self.dilation, self.normalize)
            return corr * self._scale() if self.normalize else corr
        if not (self.fmap1.is_cuda and self.fmap2.is_cuda):
            raise RuntimeError(
                "localcorr_b200 spatial correlation requires inputs on a CUDA device, but they "
                f"are on {self.fmap1.device}.")
        out = ops.spatial_corr(self.fmap1, self.fmap2, self.radius, self.dilation,
                               self._scale())
        return out.reshape(b, rd * rd, h, w)
