"""Lookups of one pyramid block share gradient accumulators.

A RAFT step calls one block many times (iterative refinement). The block
routes the lookups' fmap gradients into one pair of buffers through the C
ABI's accumulate flags and converts them once (ops.LookupGrads and
ops.LookupGradSink); these tests check that the resulting gradients equal
the per-lookup path (ops.ScaledPyramidCorr, summed by autograd) and the
float64 oracle, also across repeated backward passes and partial losses.
"""

import math

import pytest
import torch

import localcorr_b200 as lc
from localcorr_b200 import ops
from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")


def _inputs(dtype, b=2, c=64, h=24, w=40, n=3, seed=0):
    f1, f2 = oracle.make_fmaps(b, c, h, w, seed=seed)
    coords = [oracle.make_coords_uniform(b, h, w, 6.0, seed=seed + 1 + i) for i in range(n)]
    g = torch.Generator().manual_seed(seed + 7)
    grads = [torch.randn(b, 4 * 81, h, w, generator=g) for _ in range(n)]
    if dtype == torch.float16:
        f1, f2 = f1.half().float(), f2.half().float()
        coords = [c_.half().float() for c_ in coords]
        grads = [g_.half().float() for g_ in grads]
    return f1, f2, coords, grads


def _fused(f1, f2, coords, grads, dtype, passes=1):
    x1 = f1.to(DEV, dtype).requires_grad_(True)
    x2 = f2.to(DEV, dtype).requires_grad_(True)
    block = lc.get_localcorr_block(x1, x2, num_levels=4, radius=4)
    outs = [block(co.to(DEV, dtype)) for co in coords]
    for i in range(passes):
        torch.autograd.backward(outs, [g.to(DEV, dtype) for g in grads], retain_graph=i + 1 < passes)
    return x1.grad.float(), x2.grad.float()


def _per_lookup(f1, f2, coords, grads, dtype):
    x1 = f1.to(DEV, dtype).requires_grad_(True)
    x2 = f2.to(DEV, dtype).requires_grad_(True)
    fm1 = ops.NchwToNhwc.apply(x1)
    packed = ops.PyramidBuild.apply(x2, 4)
    b, c, h, w = x1.shape
    outs = [ops.ScaledPyramidCorr.apply(fm1, packed, co.to(DEV, dtype), 4, 4, 1, False,
                                        1.0 / math.sqrt(c)).reshape(b, -1, h, w)
            for co in coords]
    torch.autograd.backward(outs, [g.to(DEV, dtype) for g in grads])
    return x1.grad.float(), x2.grad.float()


TOL = {torch.float32: dict(rtol=1e-5, atol=1e-4), torch.float16: dict(rtol=1e-2, atol=1e-2)}


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16], ids=["f32", "f16"])
def test_fused_lookups_match_per_lookup_and_oracle(dtype):
    f1, f2, coords, grads = _inputs(dtype)
    a1, a2 = _fused(f1, f2, coords, grads, dtype)
    b1, b2 = _per_lookup(f1, f2, coords, grads, dtype)
    torch.testing.assert_close(a1, b1, **TOL[dtype])
    torch.testing.assert_close(a2, b2, **TOL[dtype])
    # float64 oracle: the sum over lookups of the block's gradients
    r1 = torch.zeros_like(f1, dtype=torch.float64)
    r2 = torch.zeros_like(f2, dtype=torch.float64)
    for co, g in zip(coords, grads):
        _, g1, g2 = oracle.block_grads(f1, f2, co, 4, 4, g)
        r1 += g1
        r2 += g2
    torch.testing.assert_close(a1.double().cpu(), r1, **TOL[dtype])
    torch.testing.assert_close(a2.double().cpu(), r2, **TOL[dtype])


def test_fused_lookups_two_backward_passes_add_up():
    dtype = torch.float32
    f1, f2, coords, grads = _inputs(dtype, seed=3)
    a1, a2 = _fused(f1, f2, coords, grads, dtype, passes=2)
    b1, b2 = _fused(f1, f2, coords, grads, dtype, passes=1)
    torch.testing.assert_close(a1, 2 * b1, rtol=1e-5, atol=1e-4)
    torch.testing.assert_close(a2, 2 * b2, rtol=1e-5, atol=1e-4)


def test_fused_lookups_only_used_outputs_contribute():
    dtype = torch.float32
    f1, f2, coords, grads = _inputs(dtype, seed=5)
    x1 = f1.to(DEV, dtype).requires_grad_(True)
    x2 = f2.to(DEV, dtype).requires_grad_(True)
    block = lc.get_localcorr_block(x1, x2, num_levels=4, radius=4)
    outs = [block(co.to(DEV, dtype)) for co in coords]
    (outs[1] * grads[1].to(DEV)).sum().backward()
    b1, b2 = _per_lookup(f1, f2, coords[1:2], grads[1:2], dtype)
    torch.testing.assert_close(x1.grad, b1, rtol=1e-5, atol=1e-4)
    torch.testing.assert_close(x2.grad, b2, rtol=1e-5, atol=1e-4)
