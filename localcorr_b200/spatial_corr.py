"""PWC-Net spatial correlation sampler module (reference spatial_corr.py:206-376).

LocalCorrCudaPyramidSampler keeps the reference constructor contract
(kernel_size=1, stride=1, padding=0, dilation=1, dilation_patch=1 asserted;
xpu_backend in {"sycl", "triton"}) and returns [B, P, P, H, W] with
[b, dy_idx, dx_idx, h, w] order. Execution is the sm_100a spatial kernel;
the reference's device dispatch (CUDA library / Triton / SYCL) is replaced
by that single engine.
"""

import torch
import torch.nn as nn

from . import _lib, ops


def get_sycl_xpu_extension():
    """The reference's torch.xpu extension loader (spatial_corr.py:100-128);
    there is no XPU engine here, so this always returns None."""
    return None


class LocalCorrCudaPyramidSampler(nn.Module):
    def __init__(self, kernel_size: int = 1, patch_size: int = 9, stride: int = 1,
                 padding: int = 0, dilation: int = 1, dilation_patch: int = 1,
                 onnx_generic: bool = False, xpu_backend: str = "sycl") -> None:
        super().__init__()
        assert kernel_size == 1, "Only kernel_size=1 is supported."
        assert stride == 1, "Only stride=1 is supported."
        assert padding == 0, "Only padding=0 is supported."
        assert dilation == 1, "Only dilation=1 is supported."
        assert dilation_patch == 1, "Only dilation_patch=1 is supported."
        assert xpu_backend in ("sycl", "triton"), f"Unknown xpu_backend: {xpu_backend!r}"
        self.md = patch_size // 2
        self.patch_size = patch_size
        self.onnx_generic = onnx_generic
        self.xpu_backend = xpu_backend
        self._coords = None

    def _identity_coords(self, b, h, w, dtype, device):
        if (self._coords is None or self._coords.shape[0] != b or self._coords.shape[2] != h
                or self._coords.shape[3] != w or self._coords.dtype != dtype
                or self._coords.device != device):
            self._coords = ops.identity_coords(b, h, w, dtype, device)
        return self._coords

    def forward(self, input1: torch.Tensor, input2: torch.Tensor) -> torch.Tensor:
        b, c, h, w = input1.shape
        if torch.onnx.is_in_onnx_export():
            from .blocks import LocalCorrCudaPyramidSpatialOnnx

            fmap1 = input1.permute(0, 2, 3, 1).contiguous()
            fmap2 = input2.permute(0, 2, 3, 1).contiguous()
            coords = self._identity_coords(b, h, w, input1.dtype, input1.device)
            corr = LocalCorrCudaPyramidSpatialOnnx.apply(fmap1, fmap2, coords, self.md, 1, None)
            return corr.view(b, self.patch_size, self.patch_size, h, w)
        if not (input1.is_cuda and input2.is_cuda):
            raise RuntimeError(
                "localcorr_b200 spatial correlation requires inputs on a CUDA device, but they "
                f"are on {input1.device}.")
        _lib.require_library()
        out = ops.spatial_corr(input1, input2, self.md, 1, 1.0)
        return out.view(b, self.patch_size, self.patch_size, h, w)
