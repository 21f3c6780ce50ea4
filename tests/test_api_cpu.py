"""Host-side behaviour of the public API (no GPU): mode dispatch, block
attributes, error behaviour on CPU tensors and a missing library, ONNX
wrappers, backend flag. Mirrors the reference's CPU suite
(tests/test_blocks.py, tests/test_localcorr_sampler.py)."""

import pytest
import torch

import localcorr_b200 as lc
from localcorr_b200 import _lib, blocks, ops
from oracle import oracle

B, C, H, W = 2, 8, 16, 24
LEVELS, RADIUS = 3, 2


@pytest.fixture
def fmaps():
    return oracle.make_fmaps(B, C, H, W, seed=20)


@pytest.mark.parametrize(
    "mode,cls",
    [
        ("localcorr_triton", blocks.LocalCorrTritonFusedBlock),
        ("localcorr_cuda", blocks.LocalCorrCudaPyramidBlock),
        ("localcorr_onnx", blocks.LocalCorrOnnxBlock),
        ("localcorr_sycl", blocks.LocalCorrSyclBlock),
        ("localcorr_auto", blocks.LocalCorrCudaPyramidBlock),
    ],
)
def test_block_dispatch_and_attributes(fmaps, mode, cls):
    block = lc.get_localcorr_block(*fmaps, num_levels=LEVELS, radius=RADIUS, corr_mode=mode)
    assert type(block) is cls
    assert block.num_levels == LEVELS and block.radius == RADIUS and block.dim == C


def test_mode_is_case_insensitive(fmaps):
    assert type(lc.get_localcorr_block(*fmaps, corr_mode="LOCALCORR_CUDA")) is \
        blocks.LocalCorrCudaPyramidBlock


def test_unknown_mode_raises(fmaps):
    with pytest.raises(ValueError, match="Unknown local corr_mode"):
        lc.get_localcorr_block(*fmaps, corr_mode="allpairs_local")
    with pytest.raises(ValueError, match="Unknown local corr_mode"):
        lc.get_localcorr_sampler(corr_mode="allpairs_spatial")


def test_onnx_flag(fmaps):
    assert lc.get_localcorr_block(*fmaps, corr_mode="localcorr_onnx").onnx_generic is True
    assert lc.get_localcorr_block(*fmaps, corr_mode="localcorr_cuda").onnx_generic is False


def test_block_on_cpu_raises_at_call(fmaps):
    block = lc.get_localcorr_block(*fmaps, num_levels=LEVELS, radius=RADIUS,
                                   corr_mode="localcorr_cuda")
    coords = oracle.make_coords_uniform(B, H, W, 3.0)
    with pytest.raises(RuntimeError, match="CUDA device"):
        block(coords)


@pytest.mark.parametrize("mode", ["localcorr_cuda", "localcorr_triton", "localcorr_onnx",
                                  "localcorr_sycl", "localcorr_auto"])
def test_sampler_dispatch_and_cpu_error(fmaps, mode):
    s = lc.get_localcorr_sampler(patch_size=9, corr_mode=mode)
    assert s.md == 4 and s.patch_size == 9
    with pytest.raises(RuntimeError, match="CUDA device"):
        s(*fmaps)


def test_pyramid_sampler_asserts():
    with pytest.raises(AssertionError):
        lc.LocalCorrCudaPyramidSampler(dilation_patch=2)
    with pytest.raises(AssertionError):
        lc.LocalCorrCudaPyramidSampler(xpu_backend="cuda")
    with pytest.raises(AssertionError):
        lc.LocalCorrCudaSpatialSampler(kernel_size=3)


def test_missing_library_raises_import_error(monkeypatch):
    monkeypatch.setattr(_lib, "_LIB", None)
    monkeypatch.setattr(_lib, "_LIB_LOADED", True)
    assert lc.get_cuda_pyramid_library() is None
    with pytest.raises(ImportError, match="localcorr_b200.csrc.build"):
        _lib.require_library()


def test_load_library_from_missing_path_returns_none(tmp_path):
    assert _lib.load_library(tmp_path / "nope.so") is None


def test_onnx_wrappers_forward_shapes():
    fmap1 = torch.zeros(B, H, W, C)
    packed = torch.zeros(B, C * H * W)
    coords = torch.zeros(B, 2, H, W)
    out = lc.LocalCorrCudaPyramidOnnx.apply(fmap1, packed, coords, RADIUS, LEVELS)
    assert out.shape == (B, LEVELS, 25, H, W) and out.dtype == fmap1.dtype
    out = lc.LocalCorrCudaPyramidSpatialOnnx.apply(fmap1, fmap1, coords, RADIUS, 2, "sqrt")
    assert out.shape == (B, 25, H, W)


def test_backend_flag():
    assert lc.get_onnx_backend() == "tensorrt"
    lc.set_onnx_backend("onnx")
    assert lc.get_onnx_backend() == "onnx"
    with pytest.raises(ValueError):
        lc.set_onnx_backend("tflite")


def test_level_geometry():
    assert ops.level_shapes(135, 240, 4) == [(135, 240), (67, 120), (33, 60), (16, 30)]
    assert ops.packed_row_elems(256, 135, 240, 4) == 256 * (32400 + 8040 + 1980 + 480)


def test_public_names_importable():
    for name in lc.__all__:
        assert hasattr(lc, name), name


def test_spatial_block_cpu_raises():
    f1, f2 = oracle.make_fmaps(1, 4, 8, 8, seed=26)
    block = lc.LocalCorrCudaPyramidSpatialBlock(f1, f2, radius=1)
    with pytest.raises(RuntimeError, match="CUDA device"):
        block()
