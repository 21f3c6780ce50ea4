"""A real enqueue of the relinked TensorRT plugin call (see
tests/test_relink_cpu.py): the node's output equals the library's own
forward on the same inputs, in float16 and float32."""

import math
import shutil

import pytest
import torch

from localcorr_b200 import _lib, ops
from oracle import oracle
from test_relink_cpu import load_relink

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def relink(tmp_path_factory):
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    if shutil.which("g++") is None:
        pytest.skip("g++ not available")
    assert _lib.load_library() is not None
    return load_relink(tmp_path_factory.mktemp("relink_gpu"))


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32], ids=["f16", "f32"])
def test_relinked_plugin_enqueue_matches_library_forward(relink, dtype):
    b, c, h, w, levels, r = 2, 128, 36, 52, 4, 4
    f1, f2 = oracle.make_fmaps(b, c, h, w, seed=81)
    co = oracle.make_coords_gauss_oob(b, h, w, 6.0, 0.05, seed=82).to(dtype).to(DEV)
    fm1 = ops.nchw_to_nhwc(f1.to(dtype).to(DEV))
    packed = ops.pyramid_build(f2.to(dtype).to(DEV), levels)
    out = torch.empty((b, levels, (2 * r + 1) ** 2, h, w), dtype=dtype, device=DEV)
    stream = torch.cuda.current_stream().cuda_stream
    rc = relink.relink_enqueue(fm1.data_ptr(), packed.data_ptr(), co.data_ptr(), out.data_ptr(),
                               b, h, w, c, 1 if dtype == torch.float16 else 0, r, levels, 1, 0,
                               stream)
    assert rc == 0, _lib.last_error()
    want = ops.pyramid_corr_forward(fm1, packed, co, r, levels, 1, False, 1.0)
    torch.cuda.synchronize()
    assert torch.equal(out, want)
    ref = oracle.pyramid_corr(f1.to(dtype).float(), f2.to(dtype).float(), co.float().cpu(),
                              levels, r)
    tol = dict(rtol=1e-2, atol=1e-2) if dtype == torch.float16 else dict(rtol=1e-5, atol=1e-4)
    s = 1.0 / math.sqrt(c)
    torch.testing.assert_close(out.double().cpu() * s, ref * s, **tol)
