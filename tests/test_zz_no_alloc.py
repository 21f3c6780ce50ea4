"""The allocation-free forward entry point, checked through the C ABI.

launchLocalCorrB200PyramidForwardNoAlloc exists for callers that may not
allocate device memory while they run (a TensorRT plugin's enqueue, work
recorded during CUDA graph capture, runtimes that reserve their memory at
start-up). It must give the same correlation as the workspace-taking entry
point launchLocalCorrB200PyramidForward on the tensor-core engine, call after
call, although every call reuses the same fixed scratch array.

This file is collected last on purpose; it also passes when run on its own
in a fresh process.
"""

import math

import pytest
import torch

from localcorr_b200 import _lib, ops
from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    handle = _lib.load_library()
    assert handle is not None, "liblocalcorr_b200.so must be built"
    return handle


def _case(seed, b=1, c=256, h=40, w=52, levels=4):
    f1, f2 = oracle.make_fmaps(b, c, h, w, seed=seed)
    coords = oracle.make_coords_gauss_oob(b, h, w, 6.0, 0.05, seed=seed + 1).half().to(DEV)
    fm1 = ops.nchw_to_nhwc(f1.half().to(DEV))
    packed = ops.pyramid_build(f2.half().to(DEV), levels)
    return fm1, packed, coords


def _no_alloc(lib, fm1, packed, coords, radius, levels, scale):
    b, h, w, c = fm1.shape
    rd = 2 * radius + 1
    out = torch.empty((b, levels, rd * rd, h, w), dtype=torch.float16, device=DEV)
    stream = torch.cuda.current_stream().cuda_stream
    ok = lib.launchLocalCorrB200PyramidForwardNoAlloc(
        fm1.data_ptr(), packed.data_ptr(), coords.data_ptr(), out.data_ptr(), b, h, w, c,
        radius, levels, _lib.F16, _lib.F16, False, scale, stream)
    return ok, out


def test_no_alloc_matches_workspace_forward_twice(lib):
    lib.localCorrB200DeviceStatus(1)
    radius, levels = 4, 4
    scale = 1.0 / math.sqrt(256)
    # Two calls in a row with different inputs: the shared scratch keeps the
    # previous call's contents, which must not leak into the next result.
    for seed in (3, 17):
        fm1, packed, coords = _case(seed)
        ok, out = _no_alloc(lib, fm1, packed, coords, radius, levels, scale)
        assert ok, _lib.last_error(lib)
        ref = ops.pyramid_corr_forward(fm1, packed, coords, radius, levels, 1, False, scale,
                                       _lib.ENGINE_TC)
        torch.cuda.synchronize()
        torch.testing.assert_close(out.float(), ref.float(), rtol=1e-2, atol=1e-2)
    assert lib.localCorrB200DeviceStatus(1) == 0


def test_no_alloc_full_size_image_fits(lib):
    # One 135x240 image of the training configuration fits the fixed scratch.
    fm1, packed, coords = _case(5, h=135, w=240)
    ok, out = _no_alloc(lib, fm1, packed, coords, 4, 4, 1.0 / 16)
    assert ok, _lib.last_error(lib)
    ref = ops.pyramid_corr_forward(fm1, packed, coords, 4, 4, 1, False, 1.0 / 16,
                                   _lib.ENGINE_TC)
    torch.testing.assert_close(out.float(), ref.float(), rtol=1e-2, atol=1e-2)


def test_no_alloc_rejects_oversize_and_unsupported(lib):
    fm1, packed, coords = _case(7, b=4, h=135, w=240)
    ok, _ = _no_alloc(lib, fm1, packed, coords, 4, 4, 1.0)
    assert not ok
    assert "bytes of scratch" in _lib.last_error(lib)
    f32 = torch.zeros(1, 8, 8, 64, device=DEV)
    out = torch.empty(1, 1, 81, 8, 8, device=DEV)
    ok = lib.launchLocalCorrB200PyramidForwardNoAlloc(
        f32.data_ptr(), f32.data_ptr(), f32.data_ptr(), out.data_ptr(), 1, 8, 8, 64, 4, 1,
        _lib.F32, _lib.F32, False, 1.0, torch.cuda.current_stream().cuda_stream)
    assert not ok and "tensor-core" in _lib.last_error(lib)


def test_no_alloc_leaves_device_memory_untouched(lib):
    # After a first call (which may load the library's device code), further
    # calls take no device memory: the free byte count of the device stays
    # the same across a call and its completion.
    fm1, packed, coords = _case(11)
    radius, levels = 4, 4
    b, h, w, c = fm1.shape
    out = torch.empty((b, levels, 81, h, w), dtype=torch.float16, device=DEV)
    stream = torch.cuda.current_stream().cuda_stream

    def call():
        return lib.launchLocalCorrB200PyramidForwardNoAlloc(
            fm1.data_ptr(), packed.data_ptr(), coords.data_ptr(), out.data_ptr(), b, h, w, c,
            radius, levels, _lib.F16, _lib.F16, False, 1.0 / 16, stream)

    assert call(), _lib.last_error(lib)
    torch.cuda.synchronize()
    free_before, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        assert call(), _lib.last_error(lib)
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info()
    assert free_after == free_before


def test_no_alloc_rejects_levels_beyond_four(lib):
    fm1, packed, coords = _case(13, levels=4)
    b, h, w, c = fm1.shape
    out = torch.empty((b, 5, 81, h, w), dtype=torch.float16, device=DEV)
    ok = lib.launchLocalCorrB200PyramidForwardNoAlloc(
        fm1.data_ptr(), packed.data_ptr(), coords.data_ptr(), out.data_ptr(), b, h, w, c, 4, 5,
        _lib.F16, _lib.F16, False, 1.0, torch.cuda.current_stream().cuda_stream)
    assert not ok
    assert "levels must be in [1, 4]" in _lib.last_error(lib)


def test_no_alloc_records_under_cuda_graph_capture(lib):
    # After one call on the device (module loaded, kernel attributes set),
    # the entry point can be recorded into a CUDA graph: it allocates
    # nothing and makes no synchronising call. The replay reads the inputs'
    # current contents.
    lib.localCorrB200DeviceStatus(1)
    radius, levels, scale = 4, 4, 1.0 / 16.0
    fm1, packed, coords = _case(5)
    b, h, w, c = fm1.shape
    out = torch.empty((b, levels, 81, h, w), dtype=torch.float16, device=DEV)
    ok, _ = _no_alloc(lib, fm1, packed, coords, radius, levels, scale)  # warm-up
    assert ok, _lib.last_error(lib)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        with torch.cuda.graph(graph, stream=side):
            ok = lib.launchLocalCorrB200PyramidForwardNoAlloc(
                fm1.data_ptr(), packed.data_ptr(), coords.data_ptr(), out.data_ptr(), b, h, w,
                c, radius, levels, _lib.F16, _lib.F16, False, scale,
                torch.cuda.current_stream().cuda_stream)
    assert ok, _lib.last_error(lib)
    torch.cuda.current_stream().wait_stream(side)
    for seed in (11, 23):
        f2m, p2, co2 = _case(seed)
        fm1.copy_(f2m)
        packed.copy_(p2)
        coords.copy_(co2)
        graph.replay()
        ref = ops.pyramid_corr_forward(fm1, packed, coords, radius, levels, 1, False, scale,
                                       _lib.ENGINE_TC)
        torch.cuda.synchronize()
        torch.testing.assert_close(out.float(), ref.float(), rtol=1e-2, atol=1e-2)
    del graph
    assert lib.localCorrB200DeviceStatus(1) == 0
