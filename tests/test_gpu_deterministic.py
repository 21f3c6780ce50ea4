"""Deterministic mode: bitwise-repeatable results from both engines.

``compute-sanitizer`` (racecheck) is closed on this pool, so races in the
scattered grad_fmap2 reduction are caught the other way round: in
deterministic mode the pixel sort orders every bin by pixel index and every
grad_fmap2 position gets exactly one add per call, so repeated calls on the
same inputs must return identical bits; a race (two writers of one position,
or an order that depends on timing) shows up as a difference. The results
must also equal the default mode's within the float16 contract (rtol/atol
1e-2), which the oracle pins elsewhere, and the oracle directly here.

The reference has no deterministic mode: its backward adds grad_fmap2 with
float atomics (cuda_pyramid/localcorr_cuda_pyramid_kernel.cu:909-916).
"""

import math

import pytest
import torch

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


@pytest.fixture(autouse=True)
def _mode_off_after():
    lib = _lib.load_library()
    lib.localCorrB200DeviceStatus(1)
    yield
    lc.set_deterministic(False)
    assert lib.localCorrB200DeviceStatus(1) == 0, "a tensor-core pipeline wait timed out"


def _inputs(b, c, h, w, levels, kind, seed):
    f1, f2 = oracle.make_fmaps(b, c, h, w, seed=seed)
    f1, f2 = f1.half(), f2.half()
    if kind == "uniform64":
        co = oracle.make_coords_uniform(b, h, w, 64.0, seed=seed + 1)
    elif kind == "converge":
        g = torch.Generator().manual_seed(seed + 1)
        co = torch.empty(b, 2, h, w)
        co[:, 0] = w / 2 + torch.rand(b, h, w, generator=g) * 3
        co[:, 1] = h / 2 + torch.rand(b, h, w, generator=g) * 3
    else:
        co = oracle.make_coords_gauss_oob(b, h, w, 6.0, 0.05, seed=seed + 1)
    fm1 = ops.nchw_to_nhwc(f1.to(DEV))
    packed = ops.pyramid_build(f2.to(DEV), levels)
    return f1, f2, co.half(), fm1, packed


def _call(fm1, packed, co, gout, r, levels, scale):
    out = ops.pyramid_corr_forward(fm1, packed, co, r, levels, 1, False, scale, _lib.ENGINE_TC)
    g1, g2 = ops.pyramid_corr_backward(fm1, packed, co, gout, r, levels, 1, False, scale,
                                       _lib.ENGINE_TC)
    return out, g1, g2


CASES = [
    # b, c, h, w, levels, radius, flow: crowded coarse levels and one overfull cell
    (4, 128, 64, 128, 4, 4, "uniform64"),
    (2, 256, 48, 80, 4, 3, "gauss_oob"),
    (2, 128, 40, 64, 4, 8, "uniform64"),
    (1, 64, 32, 48, 3, 4, "converge"),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "b{}c{}_{}x{}_l{}r{}_{}".format(*c))
def test_deterministic_mode_repeats_bitwise(case):
    b, c, h, w, levels, r, kind = case
    f1, f2, co, fm1, packed = _inputs(b, c, h, w, levels, kind, seed=31)
    rd = 2 * r + 1
    scale = 1.0 / math.sqrt(c)
    gout = torch.randn(b, levels, rd * rd, h, w,
                       generator=torch.Generator().manual_seed(32)).half().to(DEV)
    cod = co.to(DEV)
    ref = _call(fm1, packed, cod, gout, r, levels, scale)  # default mode
    lc.set_deterministic(True)
    assert _lib.load_library().localCorrB200GetDeterministic() == 1
    first = _call(fm1, packed, cod, gout, r, levels, scale)
    for _ in range(3):
        again = _call(fm1, packed, cod, gout, r, levels, scale)
        for x, y in zip(first, again):
            assert torch.equal(x, y)
    for x, y in zip(first, ref):
        torch.testing.assert_close(x.float(), y.float(), **F16TOL)
    if b * h * w <= 4096:
        x1 = f1.double().requires_grad_(True)
        x2 = f2.double().requires_grad_(True)
        o = oracle.pyramid_corr(x1, x2, co.double(), levels, r) * scale
        torch.testing.assert_close(first[0].double().cpu(), o.detach(), **F16TOL)
        e1, e2 = torch.autograd.grad(o, [x1, x2], gout.double().cpu())
        torch.testing.assert_close(first[1].permute(0, 3, 1, 2).double().cpu(), e1, **F16TOL)
        g2n = ops.pyramid_build_backward(first[2], (b, c, h, w), levels, torch.float32)
        torch.testing.assert_close(g2n.double().cpu(), e2, **F16TOL)


def test_torch_deterministic_flag_turns_the_mode_on():
    lib = _lib.load_library()
    b, c, h, w, levels, r = 1, 64, 24, 32, 2, 4
    _, _, co, fm1, packed = _inputs(b, c, h, w, levels, "gauss_oob", seed=41)
    torch.use_deterministic_algorithms(True)
    try:
        ops.pyramid_corr_forward(fm1, packed, co.to(DEV), r, levels)
        assert lib.localCorrB200GetDeterministic() == 1
    finally:
        torch.use_deterministic_algorithms(False)
    ops.pyramid_corr_forward(fm1, packed, co.to(DEV), r, levels)
    assert lib.localCorrB200GetDeterministic() == 0


def test_block_training_step_repeats_bitwise():
    # the block's autograd path: forward keeps the sort, the backward reuses
    # it and accumulates both gradients over the lookups
    b, c, h, w, levels, r = 2, 128, 40, 56, 4, 4
    f1, f2 = oracle.make_fmaps(b, c, h, w, seed=51)
    co = [oracle.make_coords_gauss_oob(b, h, w, 6.0, 0.05, seed=52 + i).to(DEV) for i in range(3)]

    def step():
        x1 = f1.half().to(DEV).requires_grad_(True)
        x2 = f2.half().to(DEV).requires_grad_(True)
        blk = lc.get_localcorr_block(x1, x2, num_levels=levels, radius=r,
                                     corr_mode="localcorr_cuda")
        loss = sum((blk(cc).float() * (i + 1)).square().mean() for i, cc in enumerate(co))
        return torch.autograd.grad(loss, [x1, x2])

    lc.set_deterministic(True)
    a = step()
    for _ in range(2):
        bb = step()
        assert torch.equal(a[0], bb[0]) and torch.equal(a[1], bb[1])


@pytest.mark.parametrize("case", [(1, 32, 16, 20, 2, 3, torch.float32),
                                  (2, 24, 23, 31, 4, 4, torch.float32),
                                  (1, 33, 18, 26, 3, 4, torch.float16)],
                         ids=lambda c: "b{}c{}_{}x{}_l{}r{}_{}".format(
                             *c[:6], str(c[6]).split(".")[-1]))
def test_cuda_core_backward_deterministic(case):
    # float32 maps (or a channel count the tensor cores do not take): the
    # CUDA-core backward without scattered atomics, grad_fmap2 pulled over
    # the sorted pixels
    b, c, h, w, levels, r, dt = case
    f1, f2 = oracle.make_fmaps(b, c, h, w, seed=61)
    fm1 = ops.nchw_to_nhwc(f1.to(DEV, dt))
    packed = ops.pyramid_build(f2.to(DEV, dt), levels)
    co = oracle.make_coords_gauss_oob(b, h, w, 5.0, 0.1, seed=62).to(DEV, dt)
    rd = 2 * r + 1
    gout = torch.randn(b, levels, rd * rd, h, w,
                       generator=torch.Generator().manual_seed(63)).to(DEV, dt)
    s1, s2 = ops.pyramid_corr_backward(fm1, packed, co, gout, r, levels, 1, False, 0.5)
    lc.set_deterministic(True)
    a1, a2 = ops.pyramid_corr_backward(fm1, packed, co, gout, r, levels, 1, False, 0.5)
    for _ in range(3):
        x1, x2 = ops.pyramid_corr_backward(fm1, packed, co, gout, r, levels, 1, False, 0.5)
        assert torch.equal(a1, x1) and torch.equal(a2, x2)
    tol = dict(rtol=1e-5, atol=1e-4) if dt == torch.float32 else F16TOL
    torch.testing.assert_close(a1.float(), s1.float(), **tol)
    torch.testing.assert_close(a2, s2, rtol=1e-5, atol=1e-4)
    # accumulate flag: a second call adds into the same buffers
    ops.pyramid_corr_backward(fm1, packed, co, gout, r, levels, 1, False, 0.5, out=(x1, x2),
                              accumulate=_lib.ACC_FMAP1 | _lib.ACC_FMAP2)
    torch.testing.assert_close(x2, 2 * a2, rtol=1e-5, atol=1e-4)
    xd1 = f1.double().requires_grad_(True)
    xd2 = f2.double().requires_grad_(True)
    if dt == torch.float16:
        xd1 = f1.half().double().requires_grad_(True)
        xd2 = f2.half().double().requires_grad_(True)
    o = oracle.pyramid_corr(xd1, xd2, co.double().cpu(), levels, r) * 0.5
    e1, e2 = torch.autograd.grad(o, [xd1, xd2], gout.double().cpu())
    torch.testing.assert_close(a1.permute(0, 3, 1, 2).double().cpu(), e1, **tol)
    g2n = ops.pyramid_build_backward(a2, (b, c, h, w), levels, torch.float32)
    torch.testing.assert_close(g2n.double().cpu(), e2, **tol)


def test_deterministic_mode_refuses_dilated_cuda_core_backward():
    b, c, h, w, levels, r = 1, 16, 16, 20, 2, 2
    f1, f2 = oracle.make_fmaps(b, c, h, w, seed=71)
    fm1 = ops.nchw_to_nhwc(f1.to(DEV))
    packed = ops.pyramid_build(f2.to(DEV), levels)
    co = oracle.make_coords_uniform(b, h, w, 4.0, seed=72).to(DEV)
    gout = torch.ones(b, levels, (2 * r + 1) ** 2, h, w, device=DEV)
    lc.set_deterministic(True)
    # the forward has no scattered adds and still runs
    ops.pyramid_corr_forward(fm1, packed, co, r, levels, 2)
    with pytest.raises(RuntimeError, match="deterministic"):
        ops.pyramid_corr_backward(fm1, packed, co, gout, r, levels, 2)
    lc.set_deterministic(False)
    ops.pyramid_corr_backward(fm1, packed, co, gout, r, levels, 2)
