"""localcorr_b200: B200-native (sm_100a) local correlation for optical flow.

Drop-in for the hot path of hmorimitsu/localcorr: RAFT-style on-the-fly
pyramid correlation and PWC-Net-style spatial correlation, forward and
backward, behind the reference's public names (reference __init__.py:46-114).
The kernels live in liblocalcorr_b200.so (C ABI: include/localcorr_b200.h),
built with ``python -m localcorr_b200.csrc.build``.
"""

from . import torch_ops  # noqa: F401  (registers torch.ops.localcorr.*)
from .backend import get_onnx_backend, set_onnx_backend
from .blocks import (
    LocalCorrCudaPyramidBlock,
    LocalCorrCudaPyramidFunction,
    LocalCorrCudaPyramidOnnx,
    LocalCorrCudaPyramidSpatialBlock,
    LocalCorrCudaSpatialSampler,
    LocalCorrOnnxBlock,
    LocalCorrOnnxSpatialSampler,
    LocalCorrSyclBlock,
    LocalCorrSyclSpatialSampler,
    LocalCorrTritonBlock,
    LocalCorrTritonFusedBlock,
    TritonSpatialCorrelationSampler,
    get_cuda_pyramid_library,
    get_localcorr_block,
    get_localcorr_sampler,
)
from .blocks import LocalCorrCudaPyramidSpatialOnnx
from .spatial_corr import LocalCorrCudaPyramidSampler, get_sycl_xpu_extension
from .ops import is_deterministic, set_deterministic

# The reference's Triton autograd Functions (triton/pyramid_corr.py:845-1246,
# triton/spatial_corr.py:108-207) have no counterpart: there is no Triton
# engine. The names stay importable and are None, as in the reference when
# triton is absent (reference __init__.py:70-85).
LocalCorrTriton = None
LocalCorrTritonFused = None
TritonSpatialCorrelationFunction = None

__version__ = "0.1.1"

__all__ = [
    "get_localcorr_block",
    "get_localcorr_sampler",
    "get_cuda_pyramid_library",
    "get_sycl_xpu_extension",
    "get_onnx_backend",
    "set_onnx_backend",
    "LocalCorrCudaPyramidBlock",
    "LocalCorrCudaPyramidFunction",
    "LocalCorrCudaPyramidOnnx",
    "LocalCorrCudaPyramidSpatialBlock",
    "LocalCorrCudaPyramidSpatialOnnx",
    "LocalCorrCudaPyramidSampler",
    "LocalCorrCudaSpatialSampler",
    "LocalCorrOnnxBlock",
    "LocalCorrOnnxSpatialSampler",
    "LocalCorrSyclBlock",
    "LocalCorrSyclSpatialSampler",
    "LocalCorrTritonBlock",
    "LocalCorrTritonFusedBlock",
    "LocalCorrTriton",
    "LocalCorrTritonFused",
    "TritonSpatialCorrelationFunction",
    "TritonSpatialCorrelationSampler",
    "set_deterministic",
    "is_deterministic",
]
