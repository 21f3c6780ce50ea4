"""Deferred grad_fmap2: one pull over many lookups of a block.

Each lookup's backward computes grad_fmap1 and keeps its grad_fmap2 records
(launchLocalCorrB200PyramidBackwardFmap1); one
launchLocalCorrB200PyramidBackwardFmap2Pull then sums every output tile over
the lookups (passes of up to 12) before one add into the float32 gradient
pyramid. The results must equal the per-lookup backward's (same float32
products, another order of addition: rtol/atol 1e-4 relative to the
gradient scale) and, through the block, the float64 oracle.
"""

import math

import pytest
import torch

import localcorr_b200 as lc
from localcorr_b200 import _lib, ops
from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    lib = _lib.load_library()
    lib.localCorrB200DeviceStatus(1)
    yield
    assert lib.localCorrB200DeviceStatus(1) == 0, "a tensor-core pipeline wait timed out"


def _maps(b, c, h, w, levels, seed):
    f1, f2 = oracle.make_fmaps(b, c, h, w, seed=seed)
    return ops.nchw_to_nhwc(f1.half().to(DEV)), ops.pyramid_build(f2.half().to(DEV), levels)


@pytest.mark.parametrize("n", [1, 5, 14])
def test_pull_over_lookups_matches_per_lookup_backward(n):
    b, c, h, w, levels, r = 2, 128, 40, 56, 4, 4
    fm1, packed = _maps(b, c, h, w, levels, seed=3)
    scale = 1.0 / math.sqrt(c)
    g = torch.Generator().manual_seed(4)
    coords = [oracle.make_coords_gauss_oob(b, h, w, 6.0, 0.05, seed=10 + i).half().to(DEV)
              for i in range(n)]
    grads = [torch.randn(b, levels, 81, h, w, generator=g).half().to(DEV) for _ in range(n)]
    # reference: every lookup's whole backward, accumulated
    r1 = torch.empty_like(fm1)
    r2 = torch.empty(packed.shape, dtype=torch.float32, device=DEV)
    for i in range(n):
        ops.pyramid_corr_backward(fm1, packed, coords[i], grads[i], r, levels, 1, False, scale,
                                  out=(r1, r2),
                                  accumulate=0 if i == 0 else _lib.ACC_FMAP1 | _lib.ACC_FMAP2)
    # deferred: grad_fmap1 per lookup, records kept, one pull
    nrec = ops.records_bytes(fm1, packed, r, levels)
    assert nrec > 0
    d1 = torch.empty_like(fm1)
    d2 = torch.full(packed.shape, float("nan"), dtype=torch.float32, device=DEV)
    states, recs = [], []
    for i in range(n):
        st = torch.empty(ops.sort_state_bytes(fm1, packed, r, levels), dtype=torch.uint8,
                         device=DEV)
        ops.pyramid_corr_forward(fm1, packed, coords[i], r, levels, 1, False, scale,
                                 sort_state=st)
        rec = torch.empty(nrec, dtype=torch.uint8, device=DEV)
        ops.pyramid_corr_backward_fmap1(fm1, packed, coords[i], grads[i], r, levels, scale, d1,
                                        0 if i == 0 else _lib.ACC_FMAP1, st, rec)
        states.append(st)
        recs.append(rec)
    ops.pyramid_corr_backward_fmap2_pull(fm1, d2, r, levels, scale, states, recs, 0)
    torch.cuda.synchronize()
    # same kernel; the two sorts may order a bin's pixels differently
    torch.testing.assert_close(d1.float(), r1.float(), rtol=1e-3, atol=1e-3)
    tol = 1e-4 * float(r2.abs().max())
    torch.testing.assert_close(d2, r2, rtol=1e-4, atol=tol)
    # accumulate flag: a second pull adds
    ops.pyramid_corr_backward_fmap2_pull(fm1, d2, r, levels, scale, states, recs,
                                         _lib.ACC_FMAP2)
    torch.testing.assert_close(d2, 2 * r2, rtol=1e-4, atol=2 * tol)


def test_block_with_many_lookups_defers_and_matches(monkeypatch):
    # 14 lookups of one block: 12 deferred lookups are pulled when the
    # twelfth gathers, the other two when the sink runs; against the
    # per-lookup backward (deferral off) and the oracle.
    b, c, h, w, levels, r, n = 1, 64, 24, 40, 4, 4, 14
    f1, f2 = oracle.make_fmaps(b, c, h, w, seed=21)
    f1, f2 = f1.half().float(), f2.half().float()
    coords = [oracle.make_coords_uniform(b, h, w, 6.0, seed=22 + i).half().float()
              for i in range(n)]
    g = torch.Generator().manual_seed(23)
    grads = [torch.randn(b, levels * 81, h, w, generator=g).half().float() for _ in range(n)]

    def run():
        x1 = f1.to(DEV, torch.float16).requires_grad_(True)
        x2 = f2.to(DEV, torch.float16).requires_grad_(True)
        blk = lc.get_localcorr_block(x1, x2, num_levels=levels, radius=r,
                                     corr_mode="localcorr_cuda")
        outs = [blk(co.to(DEV, torch.float16)) for co in coords]
        torch.autograd.backward(outs, [gg.to(DEV, torch.float16) for gg in grads])
        return x1.grad.float(), x2.grad.float()

    monkeypatch.setattr(ops, "DEFER_FMAP2", True)
    a1, a2 = run()
    monkeypatch.setattr(ops, "DEFER_FMAP2", False)
    b1, b2 = run()
    torch.testing.assert_close(a1, b1, rtol=1e-2, atol=1e-2)
    torch.testing.assert_close(a2, b2, rtol=1e-2, atol=1e-2)
    x1 = f1.double().requires_grad_(True)
    x2 = f2.double().requires_grad_(True)
    tot = 0
    for co, gg in zip(coords, grads):
        o = oracle.pyramid_corr(x1, x2, co.double(), levels, r) / math.sqrt(c)
        tot = tot + (o.reshape(b, -1, h, w) * gg.double()).sum()
    e1, e2 = torch.autograd.grad(tot, [x1, x2])
    torch.testing.assert_close(a1.double().cpu(), e1, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(a2.double().cpu(), e2, rtol=2e-2, atol=2e-2)
