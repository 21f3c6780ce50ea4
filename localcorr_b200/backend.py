"""ONNX-export backend selection (reference backend.py:1-59).

"tensorrt" (default) exports the correlation as the LocalCorrCudaPyramid
plugin node; "onnx" asks for standard ops, which this package does not
emit (the blocks raise NotImplementedError under export in that case).
The variable LOCALCORR_ONNX_BACKEND sets the initial value.
"""

import os

import torch

_VALID = ("tensorrt", "onnx")
_onnx_backend = os.environ.get("LOCALCORR_ONNX_BACKEND", "tensorrt").lower()
if _onnx_backend not in _VALID:
    _onnx_backend = "tensorrt"


def set_onnx_backend(backend: str) -> None:
    global _onnx_backend
    b = backend.lower()
    if b not in _VALID:
        raise ValueError(f"Unknown ONNX backend: {backend!r} (expected one of {_VALID})")
    _onnx_backend = b


def get_onnx_backend() -> str:
    return _onnx_backend


def use_onnx_generic_ops() -> bool:
    """True only while exporting with the "onnx" backend selected."""
    return torch.onnx.is_in_onnx_export() and _onnx_backend == "onnx"
