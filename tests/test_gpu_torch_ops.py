"""torch.ops.localcorr.*: the engine as registered PyTorch custom operators.

torch.library.opcheck checks each operator's schema, fake-tensor (meta)
implementation, autograd registration and AOT-dispatch behaviour against its
real CUDA kernel; torch.compile(fullgraph=True) traces the public block API
(inference and training) without a graph break and matches eager execution
and the oracle.
"""

import math

import pytest
import torch
from torch.library import opcheck

import localcorr_b200 as lc
from localcorr_b200 import _lib, ops
from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda"
F16TOL = dict(rtol=1e-2, atol=1e-2)


@pytest.fixture(scope="module", autouse=True)
def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    assert _lib.load_library() is not None


def _maps(dtype, b=1, c=64, h=20, w=28, seed=0):
    f1, f2 = oracle.make_fmaps(b, c, h, w, seed=seed)
    co = oracle.make_coords_uniform(b, h, w, 6.0, seed=seed + 1)
    return f1.to(DEV, dtype), f2.to(DEV, dtype), co.to(DEV, dtype)


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32], ids=["f16", "f32"])
def test_opcheck_layout_and_pyramid_ops(dtype):
    f1, f2, co = _maps(dtype)
    opcheck(torch.ops.localcorr.nchw_to_nhwc.default, (f1.requires_grad_(True),))
    nhwc = ops.nchw_to_nhwc(f1.detach())
    opcheck(torch.ops.localcorr.nhwc_to_nchw.default, (nhwc.requires_grad_(True),))
    opcheck(torch.ops.localcorr.pyramid_build.default, (f2.requires_grad_(True), 3))
    packed = ops.pyramid_build(f2.detach(), 3)
    opcheck(torch.ops.localcorr.pyramid_build_backward.default,
            (torch.randn_like(packed), 1, 64, 20, 28, 3, dtype))


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32], ids=["f16", "f32"])
def test_opcheck_pyramid_corr(dtype):
    f1, f2, co = _maps(dtype, c=64)
    fm1 = ops.nchw_to_nhwc(f1).requires_grad_(True)
    packed = ops.pyramid_build(f2, 3).requires_grad_(True)
    args = (fm1, packed, co, 3, 3, 1, False, 0.125, 0, 0)
    opcheck(torch.ops.localcorr.pyramid_corr.default, args)
    g = torch.randn(1, 3, 49, 20, 28, device=DEV, dtype=dtype)
    opcheck(torch.ops.localcorr.pyramid_corr_backward.default,
            (fm1.detach(), packed.detach(), co, g, 3, 3, 1, False, 0.125, 0, 0))


def test_opcheck_spatial_corr():
    f1, f2, _ = _maps(torch.float32, c=32)
    opcheck(torch.ops.localcorr.spatial_corr.default,
            (f1.requires_grad_(True), f2.requires_grad_(True), 4, 1, 1.0))
    g = torch.randn(1, 9, 9, 20, 28, device=DEV)
    opcheck(torch.ops.localcorr.spatial_corr_backward.default,
            (f1.detach(), f2.detach(), g, 4, 1, 1.0))


def test_pyramid_corr_op_matches_oracle_and_grads():
    f1, f2, co = _maps(torch.float16, c=128, h=24, w=40)
    x1 = f1.detach().requires_grad_(True)
    x2 = f2.detach().requires_grad_(True)
    fm1 = torch.ops.localcorr.nchw_to_nhwc(x1)
    packed = torch.ops.localcorr.pyramid_build(x2, 4)
    out = torch.ops.localcorr.pyramid_corr(fm1, packed, co, 4, 4, 1, False,
                                           1 / math.sqrt(128), 0, 0)
    gout = torch.randn(out.shape, generator=torch.Generator().manual_seed(5)).half()
    out.backward(gout.to(DEV))
    ref, e1, e2 = oracle.block_grads(f1.float().cpu(), f2.float().cpu(), co.float().cpu(), 4, 4,
                                     gout.float().reshape(1, -1, 24, 40))
    torch.testing.assert_close(out.double().cpu().reshape(ref.shape), ref, **F16TOL)
    torch.testing.assert_close(x1.grad.double().cpu(), e1, **F16TOL)
    torch.testing.assert_close(x2.grad.double().cpu(), e2, **F16TOL)


def _block_call(f1, f2, co):
    block = lc.get_localcorr_block(f1, f2, num_levels=4, radius=4, corr_mode="localcorr_cuda")
    return block(co) + block(co + 0.5)


def test_compile_fullgraph_block_inference():
    f1, f2, co = _maps(torch.float16, c=128, h=24, w=40, seed=3)
    with torch.no_grad():
        eager = _block_call(f1, f2, co)
        compiled = torch.compile(_block_call, fullgraph=True)(f1, f2, co)
    torch.testing.assert_close(compiled, eager, rtol=0, atol=0)


def test_compile_fullgraph_block_training():
    torch._dynamo.reset()
    f1, f2, co = _maps(torch.float16, c=128, h=24, w=40, seed=4)
    gout = torch.randn(1, 324, 24, 40, generator=torch.Generator().manual_seed(6)).half().to(DEV)

    def step(a, b, c):
        return (_block_call(a, b, c).float() * gout.float()).sum()

    grads = []
    for fn in (step, torch.compile(step, fullgraph=True)):
        x1 = f1.detach().requires_grad_(True)
        x2 = f2.detach().requires_grad_(True)
        loss = fn(x1, x2, co)
        loss.backward()
        grads.append((loss.detach(), x1.grad, x2.grad))
    (l0, a1, a2), (l1, b1, b2) = grads
    torch.testing.assert_close(l1, l0, rtol=1e-3, atol=1e-2)
    torch.testing.assert_close(b1.float(), a1.float(), **F16TOL)
    torch.testing.assert_close(b2.float(), a2.float(), **F16TOL)


def test_compile_fullgraph_sampler():
    f1, f2, _ = _maps(torch.float32, c=32, seed=7)
    sampler = lc.get_localcorr_sampler(patch_size=9, corr_mode="localcorr_cuda")
    eager = sampler(f1, f2)
    compiled = torch.compile(lambda a, b: sampler(a, b), fullgraph=True)(f1, f2)
    torch.testing.assert_close(compiled, eager, rtol=0, atol=0)
