"""Tensor-level wrappers of the C ABI and their autograd Functions.

Every op launches on torch's current CUDA stream of the input's device and
allocates its outputs (and any engine workspace) from torch's caching
allocator. Inputs must be CUDA tensors of dtype float32 or float16; there is
no CPU fallback.
"""

from __future__ import annotations

import ctypes
import math
import os

import torch

from . import _lib

_DTYPES = {torch.float32: _lib.F32, torch.float16: _lib.F16}


def _dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPES[t.dtype]
    except KeyError:
        raise RuntimeError(
            f"localcorr_b200 requires float32 or float16 tensors, but got {t.dtype}."
        ) from None


def _require_cuda(*tensors: torch.Tensor, what: str = "localcorr_b200") -> None:
    for t in tensors:
        if not t.is_cuda:
            raise RuntimeError(
                f"{what} requires tensors on a CUDA device, but got a tensor on {t.device}."
            )


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


# Optional launch timer: a list that receives (name, start_event, end_event)
# for every engine call, recorded on the launching (current) stream. Used by
# bench.py to time the dominant kernel live inside its timed region.
_timer = None


def set_launch_timer(records):
    """Install (a list) or remove (None) the engine-call timer."""
    global _timer
    _timer = records


def _timed(name, fn, nbytes=None):
    """Run fn; with the timer installed, record (name, start, end, nbytes)
    around it (nbytes: the call's algorithmic bytes, when the caller knows)."""
    if _timer is None:
        return fn()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    res = fn()
    end.record()
    _timer.append((name, start, end, nbytes))
    return res


def level_shapes(h: int, w: int, levels: int) -> list[tuple[int, int]]:
    """Floor-halved level dims of the pyramid (blocks.py:371-376)."""
    return [(h >> l, w >> l) for l in range(levels)]


def packed_row_elems(c: int, h: int, w: int, levels: int) -> int:
    return sum(c * hl * wl for hl, wl in level_shapes(h, w, levels))


# ---------------------------------------------------------------------------
# raw launchers (no autograd)
# ---------------------------------------------------------------------------

def nchw_to_nhwc(x: torch.Tensor) -> torch.Tensor:
    lib = _lib.require_library()
    _require_cuda(x)
    x = x.contiguous()
    b, c, h, w = x.shape
    out = torch.empty((b, h, w, c), dtype=x.dtype, device=x.device)
    with torch.cuda.device(x.device):
        ok = lib.launchLocalCorrB200NchwToNhwc(x.data_ptr(), out.data_ptr(), b, c, h * w,
                                               _dtype_code(x), _stream(x))
    _lib.check(ok, "NCHW->NHWC transpose", lib)
    return out


def nhwc_to_nchw(x: torch.Tensor) -> torch.Tensor:
    lib = _lib.require_library()
    _require_cuda(x)
    x = x.contiguous()
    b, h, w, c = x.shape
    out = torch.empty((b, c, h, w), dtype=x.dtype, device=x.device)
    with torch.cuda.device(x.device):
        ok = lib.launchLocalCorrB200NhwcToNchw(x.data_ptr(), out.data_ptr(), b, c, h * w,
                                               _dtype_code(x), _stream(x))
    _lib.check(ok, "NHWC->NCHW transpose", lib)
    return out


def pyramid_build(fmap2: torch.Tensor, levels: int) -> torch.Tensor:
    """fmap2 [B,C,H,W] -> batch-major packed NHWC pyramid [B, C*sum h_l*w_l]."""
    lib = _lib.require_library()
    _require_cuda(fmap2)
    fmap2 = fmap2.contiguous()
    b, c, h, w = fmap2.shape
    packed = torch.empty((b, packed_row_elems(c, h, w, levels)), dtype=fmap2.dtype,
                         device=fmap2.device)
    with torch.cuda.device(fmap2.device):
        ok = lib.launchLocalCorrB200PyramidBuild(fmap2.data_ptr(), packed.data_ptr(), b, c, h,
                                                 w, levels, _dtype_code(fmap2), _stream(fmap2))
    _lib.check(ok, "pyramid build", lib)
    return packed


def pyramid_build_backward(grad_packed: torch.Tensor, shape, levels: int,
                           dtype: torch.dtype) -> torch.Tensor:
    lib = _lib.require_library()
    grad_packed = grad_packed.contiguous()
    b, c, h, w = shape
    out = torch.empty((b, c, h, w), dtype=dtype, device=grad_packed.device)
    is_f32 = grad_packed.dtype == torch.float32
    if not is_f32 and grad_packed.dtype != dtype:
        grad_packed = grad_packed.to(dtype)
    with torch.cuda.device(grad_packed.device):
        ok = lib.launchLocalCorrB200PyramidBuildBackward(
            grad_packed.data_ptr(), is_f32, out.data_ptr(), b, c, h, w, levels,
            _DTYPES[dtype], _stream(grad_packed))
    _lib.check(ok, "pyramid build backward", lib)
    return out


def workspace_bytes(b, h, w, c, radius, levels, dilation, dtype_code, engine,
                    map_hw=None) -> int:
    lib = _lib.require_library()
    if map_hw is not None:
        return int(lib.localCorrB200PyramidWorkspaceBytesMapDims(
            b, h, w, map_hw[0], map_hw[1], c, radius, levels, dilation, dtype_code, engine))
    return int(lib.localCorrB200PyramidWorkspaceBytes(b, h, w, c, radius, levels, dilation,
                                                      dtype_code, engine))


def sort_state_bytes(fmap1, fmap2_packed, radius, levels, dilation=1, engine=_lib.ENGINE_AUTO,
                     map_hw=None) -> int:
    """Bytes of the pixel-sort state a forward can keep for its backward
    (``localCorrB200PyramidSortStateBytes``; 0 on the CUDA-core engine)."""
    lib = _lib.require_library()
    b, h, w, c = fmap1.shape
    md = _map_dims(fmap1, fmap2_packed, levels, map_hw) or (h, w)
    return int(lib.localCorrB200PyramidSortStateBytes(b, h, w, md[0], md[1], c, radius, levels,
                                                      dilation, _dtype_code(fmap1), engine))


def records_bytes(fmap1, fmap2_packed, radius, levels) -> int:
    """Bytes of one lookup's kept grad_fmap2 records
    (``localCorrB200PyramidRecordsBytes``; 0 when the tensor-core engine does
    not take the configuration)."""
    lib = _lib.require_library()
    if fmap1.dtype != torch.float16:
        return 0
    b, h, w, c = fmap1.shape
    return int(lib.localCorrB200PyramidRecordsBytes(b, h, w, h, w, c, radius, levels))


def pyramid_corr_backward_fmap1(fmap1, fmap2_packed, coords, corr_grad, radius, levels, scale,
                                g1, accumulate, sort_state, records):
    """grad_fmap1 of one lookup into g1 (added when ``accumulate`` has
    ``ACC_FMAP1``), its grad_fmap2 records left in ``records`` for
    :func:`pyramid_corr_backward_fmap2_pull` (``...BackwardFmap1``)."""
    lib = _lib.require_library()
    _sync_deterministic(lib)
    b, h, w, c = fmap1.shape
    corr_grad = corr_grad.contiguous()
    if corr_grad.dtype != fmap1.dtype:
        corr_grad = corr_grad.to(fmap1.dtype)
    nbytes = workspace_bytes(b, h, w, c, radius, levels, 1, _lib.F16, _lib.ENGINE_TC)
    ws, nws = _workspace(fmap1, nbytes - sort_state.numel())
    with torch.cuda.device(fmap1.device):
        ok = _timed("pyramid_bwd", lambda: lib.launchLocalCorrB200PyramidBackwardFmap1(
            fmap1.data_ptr(), fmap2_packed.data_ptr(), coords.data_ptr(), corr_grad.data_ptr(),
            g1.data_ptr(), b, h, w, h, w, c, radius, levels, _dtype_code(coords), False,
            float(scale), int(accumulate), sort_state.data_ptr(), sort_state.numel(),
            records.data_ptr(), records.numel(), ws.data_ptr() if ws is not None else None, nws,
            _stream(fmap1)))
    _lib.check(ok, "pyramid correlation backward (grad_fmap1)", lib)


def pyramid_corr_backward_fmap2_pull(fmap1, g2, radius, levels, scale, sort_states, records,
                                     accumulate):
    """grad_fmap2 of the kept lookups into the float32 packed g2 (added when
    ``accumulate`` has ``ACC_FMAP2``) (``...BackwardFmap2Pull``)."""
    lib = _lib.require_library()
    b, h, w, c = fmap1.shape
    n = len(sort_states)
    arr = ctypes.c_void_p * max(n, 1)
    sp = arr(*[t.data_ptr() for t in sort_states])
    rp = arr(*[t.data_ptr() for t in records])
    ws = torch.empty(256, dtype=torch.uint8, device=fmap1.device)
    with torch.cuda.device(fmap1.device):
        ok = _timed("pyramid_bwd_pull", lambda: lib.launchLocalCorrB200PyramidBackwardFmap2Pull(
            sp, rp, n, g2.data_ptr(), b, h, w, h, w, c, radius, levels, float(scale),
            int(accumulate), ws.data_ptr(), ws.numel(), _stream(fmap1)))
    _lib.check(ok, "pyramid correlation backward (grad_fmap2 pull)", lib)


def _map_dims(fmap1, fmap2_packed, levels, map_hw):
    """(H2, W2) of the map behind fmap2_packed, or None when it is fmap1's grid.

    map_hw decouples the pyramid's level-0 size from fmap1's pixel grid (the
    ``...MapDims`` entry points): a row band of fmap1/coords against a whole
    frame's pyramid."""
    b, h, w, c = fmap1.shape
    if map_hw is None or (int(map_hw[0]), int(map_hw[1])) == (h, w):
        return None
    h2, w2 = int(map_hw[0]), int(map_hw[1])
    if fmap2_packed.numel() != b * packed_row_elems(c, h2, w2, levels):
        raise RuntimeError(
            f"fmap2_packed has {fmap2_packed.numel()} elements; a {levels}-level pyramid of "
            f"a {h2}x{w2} map with B={b}, C={c} has {b * packed_row_elems(c, h2, w2, levels)}")
    return h2, w2


_USER_DETERMINISTIC = False
_LIB_DETERMINISTIC = None  # the mode last pushed into the library


def set_deterministic(on: bool) -> None:
    """Deterministic mode of the library (``localCorrB200SetDeterministic``).

    The tensor-core engine then sorts pixels in a fixed order and adds every
    grad_fmap2 position once per call, so forward and backward give bitwise
    identical results on identical inputs; the CUDA-core engine's backward
    pulls grad_fmap2 over the same sort instead of scattering float atomics
    (dilation 1 and 1..4 levels; other configurations raise). The mode is
    also on while ``torch.use_deterministic_algorithms(True)`` is in effect.
    """
    global _USER_DETERMINISTIC
    _USER_DETERMINISTIC = bool(on)
    _sync_deterministic(_lib.require_library())


def is_deterministic() -> bool:
    return _USER_DETERMINISTIC or torch.are_deterministic_algorithms_enabled()


def _sync_deterministic(lib) -> None:
    global _LIB_DETERMINISTIC
    want = is_deterministic()
    if want != _LIB_DETERMINISTIC:
        lib.localCorrB200SetDeterministic(int(want))
        _LIB_DETERMINISTIC = want


def _workspace(t: torch.Tensor, nbytes: int):
    if nbytes == 0:
        return None, 0
    ws = torch.empty((nbytes + 255) // 256 * 256, dtype=torch.uint8, device=t.device)
    return ws, ws.numel()


def pyramid_corr_forward(fmap1, fmap2_packed, coords, radius, levels, dilation=1,
                         ymajor=False, scale=1.0, engine=_lib.ENGINE_AUTO,
                         map_hw=None, sort_state=None) -> torch.Tensor:
    """corr [B, L, RD^2, H, W] = scale * local correlation (extended C ABI).

    ``map_hw=(H2, W2)``: fmap2_packed is the pyramid of an H2 x W2 map while
    fmap1/coords/corr cover an H x W pixel grid (``...MapDims`` entry).
    ``sort_state``: a uint8 tensor of :func:`sort_state_bytes` bytes that
    receives the pixel sort for the backward of the same coords
    (``...ForwardKeepSort`` entry)."""
    lib = _lib.require_library()
    _sync_deterministic(lib)
    b, h, w, c = fmap1.shape
    rd = 2 * radius + 1
    dt = _dtype_code(fmap1)
    cdt = _dtype_code(coords)
    md = _map_dims(fmap1, fmap2_packed, levels, map_hw)
    corr = torch.empty((b, levels, rd * rd, h, w), dtype=fmap1.dtype, device=fmap1.device)
    nbytes = workspace_bytes(b, h, w, c, radius, levels, dilation, dt, engine, md)
    if sort_state is not None:
        md2 = md or (h, w)
        ws, nws = _workspace(fmap1, nbytes - sort_state.numel())
        with torch.cuda.device(fmap1.device):
            ok = _timed("pyramid_fwd", lambda: lib.launchLocalCorrB200PyramidForwardKeepSort(
                fmap1.data_ptr(), fmap2_packed.data_ptr(), coords.data_ptr(), corr.data_ptr(),
                b, h, w, md2[0], md2[1], c, radius, levels, dilation, dt, cdt, bool(ymajor),
                float(scale), engine, sort_state.data_ptr(), sort_state.numel(),
                ws.data_ptr() if ws is not None else None, nws, _stream(fmap1)))
        _lib.check(ok, "pyramid correlation forward", lib)
        return corr
    ws, nws = _workspace(fmap1, nbytes)
    wsp = ws.data_ptr() if ws is not None else None
    with torch.cuda.device(fmap1.device):
        if md is None:
            ok = _timed("pyramid_fwd", lambda: lib.launchLocalCorrB200PyramidForward(
                fmap1.data_ptr(), fmap2_packed.data_ptr(), coords.data_ptr(), corr.data_ptr(),
                b, h, w, c, radius, levels, dilation, dt, cdt, bool(ymajor), float(scale),
                engine, wsp, nws, _stream(fmap1)))
        else:
            ok = _timed("pyramid_fwd", lambda: lib.launchLocalCorrB200PyramidForwardMapDims(
                fmap1.data_ptr(), fmap2_packed.data_ptr(), coords.data_ptr(), corr.data_ptr(),
                b, h, w, md[0], md[1], c, radius, levels, dilation, dt, cdt, bool(ymajor),
                float(scale), engine, wsp, nws, _stream(fmap1)))
    _lib.check(ok, "pyramid correlation forward", lib)
    return corr


def pyramid_corr_backward(fmap1, fmap2_packed, coords, corr_grad, radius, levels,
                          dilation=1, ymajor=False, scale=1.0, engine=_lib.ENGINE_AUTO,
                          out=None, accumulate=0, map_hw=None, sort_state=None):
    """Returns (grad_fmap1 [B,H,W,C] dtype, grad_fmap2_packed float32).

    With ``out=(g1, g2)`` the gradients go into those buffers; ``accumulate``
    (flags ``_lib.ACC_FMAP1`` / ``_lib.ACC_FMAP2``) adds into them instead of
    overwriting. ``map_hw`` as in :func:`pyramid_corr_forward`.
    ``sort_state``: the buffer a :func:`pyramid_corr_forward` of the same
    coords filled (``...BackwardWithSort`` entry: no second sort)."""
    lib = _lib.require_library()
    _sync_deterministic(lib)
    b, h, w, c = fmap1.shape
    dt = _dtype_code(fmap1)
    cdt = _dtype_code(coords)
    md = _map_dims(fmap1, fmap2_packed, levels, map_hw)
    corr_grad = corr_grad.contiguous()
    if corr_grad.dtype != fmap1.dtype:
        corr_grad = corr_grad.to(fmap1.dtype)
    if out is not None:
        g1, g2 = out
    else:
        g1 = torch.empty_like(fmap1)
        g2 = torch.empty(fmap2_packed.shape, dtype=torch.float32, device=fmap1.device)
    nbytes = workspace_bytes(b, h, w, c, radius, levels, dilation, dt, engine, md)
    if sort_state is not None:
        md2 = md or (h, w)
        ws, nws = _workspace(fmap1, nbytes - sort_state.numel())
        with torch.cuda.device(fmap1.device):
            ok = _timed("pyramid_bwd", lambda: lib.launchLocalCorrB200PyramidBackwardWithSort(
                fmap1.data_ptr(), fmap2_packed.data_ptr(), coords.data_ptr(),
                corr_grad.data_ptr(), g1.data_ptr(), g2.data_ptr(), b, h, w, md2[0], md2[1], c,
                radius, levels, dilation, dt, cdt, bool(ymajor), float(scale), int(accumulate),
                engine, sort_state.data_ptr(), sort_state.numel(),
                ws.data_ptr() if ws is not None else None, nws, _stream(fmap1)))
        _lib.check(ok, "pyramid correlation backward", lib)
        return g1, g2
    ws, nws = _workspace(fmap1, nbytes)
    wsp = ws.data_ptr() if ws is not None else None
    with torch.cuda.device(fmap1.device):
        if md is None:
            ok = _timed("pyramid_bwd", lambda: lib.launchLocalCorrB200PyramidBackward(
                fmap1.data_ptr(), fmap2_packed.data_ptr(), coords.data_ptr(),
                corr_grad.data_ptr(), g1.data_ptr(), g2.data_ptr(), b, h, w, c, radius, levels,
                dilation, dt, cdt, bool(ymajor), float(scale), int(accumulate), engine, wsp,
                nws, _stream(fmap1)))
        else:
            ok = _timed("pyramid_bwd", lambda: lib.launchLocalCorrB200PyramidBackwardMapDims(
                fmap1.data_ptr(), fmap2_packed.data_ptr(), coords.data_ptr(),
                corr_grad.data_ptr(), g1.data_ptr(), g2.data_ptr(), b, h, w, md[0], md[1], c,
                radius, levels, dilation, dt, cdt, bool(ymajor), float(scale),
                int(accumulate), engine, wsp, nws, _stream(fmap1)))
    _lib.check(ok, "pyramid correlation backward", lib)
    return g1, g2


def spatial_forward(in1, in2, radius, dilation=1, scale=1.0) -> torch.Tensor:
    lib = _lib.require_library()
    b, c, h, w = in1.shape
    rd = 2 * radius + 1
    out = torch.empty((b, rd, rd, h, w), dtype=in1.dtype, device=in1.device)
    nbytes = (in1.numel() + in2.numel() + out.numel()) * in1.element_size()
    with torch.cuda.device(in1.device):
        ok = _timed("spatial_fwd", lambda: lib.launchLocalCorrB200SpatialForward(
            in1.data_ptr(), in2.data_ptr(), out.data_ptr(), b, c, h, w, radius, dilation,
            _dtype_code(in1), float(scale), _stream(in1)), nbytes)
    _lib.check(ok, "spatial correlation forward", lib)
    return out


def spatial_backward(in1, in2, grad_out, radius, dilation=1, scale=1.0, need1=True,
                     need2=True):
    lib = _lib.require_library()
    b, c, h, w = in1.shape
    grad_out = grad_out.contiguous()
    if grad_out.dtype != in1.dtype:
        grad_out = grad_out.to(in1.dtype)
    g1 = torch.empty_like(in1) if need1 else None
    g2 = torch.empty_like(in2) if need2 else None
    # grad_out and the inputs read, the input gradients written
    nbytes = (grad_out.numel() + (in1.numel() if need2 else 0) + (in2.numel() if need1 else 0)
              + (in1.numel() if need1 else 0) + (in2.numel() if need2 else 0)) * in1.element_size()
    with torch.cuda.device(in1.device):
        ok = _timed("spatial_bwd", lambda: lib.launchLocalCorrB200SpatialBackward(
            in1.data_ptr(), in2.data_ptr(), grad_out.data_ptr(),
            g1.data_ptr() if g1 is not None else None, g2.data_ptr() if g2 is not None else None,
            b, c, h, w, radius, dilation, _dtype_code(in1), float(scale), _stream(in1)), nbytes)
    _lib.check(ok, "spatial correlation backward", lib)
    return g1, g2


SPATIAL_KERNEL_MAX_RADIUS = 4


# ---------------------------------------------------------------------------
# autograd Functions
# ---------------------------------------------------------------------------

class NchwToNhwc(torch.autograd.Function):
    """fmap1.permute(0, 2, 3, 1).contiguous() (blocks.py:370) as one kernel."""

    @staticmethod
    def forward(ctx, x):
        return nchw_to_nhwc(x)

    @staticmethod
    def backward(ctx, g):
        return nhwc_to_nchw(g)


class PyramidBuild(torch.autograd.Function):
    """avg_pool2d pyramid + NHWC + batch-major pack (blocks.py:371-383) in one kernel."""

    @staticmethod
    def forward(ctx, fmap2, levels):
        ctx.shape = tuple(fmap2.shape)
        ctx.levels = int(levels)
        ctx.dtype = fmap2.dtype
        return pyramid_build(fmap2, int(levels))

    @staticmethod
    def backward(ctx, g):
        return pyramid_build_backward(g, ctx.shape, ctx.levels, ctx.dtype), None


class ScaledPyramidCorr(torch.autograd.Function):
    """scale * pyramid correlation, the fused form of the RAFT block call
    (blocks.py:391-411: kernel launch, then reshape and division by sqrt(C)).
    ``map_hw`` as in :func:`pyramid_corr_forward`."""

    @staticmethod
    def forward(ctx, fmap1, fmap2_packed, coords, radius, levels, dilation, ymajor, scale,
                map_hw=None):
        coords = coords.contiguous()
        corr = pyramid_corr_forward(fmap1, fmap2_packed, coords, radius, levels, dilation,
                                    ymajor, scale, map_hw=map_hw)
        ctx.save_for_backward(fmap1, fmap2_packed, coords)
        ctx.params = (int(radius), int(levels), int(dilation), bool(ymajor), float(scale))
        ctx.map_hw = map_hw
        return corr

    @staticmethod
    def backward(ctx, corr_grad):
        fmap1, fmap2_packed, coords = ctx.saved_tensors
        radius, levels, dilation, ymajor, scale = ctx.params
        g1 = g2 = None
        if ctx.needs_input_grad[0] or ctx.needs_input_grad[1]:
            g1, g2 = pyramid_corr_backward(fmap1, fmap2_packed, coords, corr_grad, radius,
                                           levels, dilation, ymajor, scale,
                                           map_hw=ctx.map_hw)
            if g2.dtype != fmap2_packed.dtype:
                g2 = g2.to(fmap2_packed.dtype)
        # RAFT detaches the sampling coordinates: zeros, as the reference
        # returns (blocks.py:534-537).
        gc = torch.zeros_like(coords) if ctx.needs_input_grad[2] else None
        return g1, g2, gc, None, None, None, None, None, None


# A block's lookups defer their grad_fmap2 to one pull over all of them
# (tensor-core engine); LOCALCORR_B200_DEFER_FMAP2=0 runs each lookup's
# whole backward instead.
DEFER_FMAP2 = os.environ.get("LOCALCORR_B200_DEFER_FMAP2", "1") not in ("0", "")


class LookupGrads:
    """Gradient accumulators shared by the lookups of one pyramid block.

    Every lookup's backward adds its fmap1 gradient (NHWC, map dtype) and its
    fmap2 gradient (packed, float32) into these buffers through the C ABI's
    accumulate flags; the first lookup of a backward pass overwrites them.
    ``LookupGradSink``'s backward, which autograd runs once after all of
    them, turns the sums into the NCHW gradients and resets the state. This
    replaces one gradient allocation, one float16 cast and one autograd
    addition per lookup and map by a single pass at the end.
    """

    # lookups whose grad_fmap2 is pulled in one pass (the kernel's limit)
    MAX_PENDING = 12

    def __init__(self, fmap1_nhwc, fmap2_packed, fmap2_shape, levels):
        self.fmap1 = fmap1_nhwc
        self.fmap2_packed = fmap2_packed
        self.fmap2_shape = tuple(fmap2_shape)
        self.levels = int(levels)
        self.g1 = None
        self.g2 = None
        # lookups whose grad_fmap2 is deferred: (sort state, records) and the
        # (radius, scale) they share
        self.pending = []
        self.pull_params = None

    def fmap1_buffer(self):
        """(g1, flag) for the next lookup's grad_fmap1."""
        if self.g1 is None:
            self.g1 = torch.empty_like(self.fmap1)
            return self.g1, 0
        return self.g1, _lib.ACC_FMAP1

    def fmap2_buffer(self):
        """(g2, flag) for the next grad_fmap2 contribution."""
        if self.g2 is None:
            self.g2 = torch.empty(self.fmap2_packed.shape, dtype=torch.float32,
                                  device=self.fmap1.device)
            return self.g2, 0
        return self.g2, _lib.ACC_FMAP2

    def buffers(self):
        """(g1, g2, flags) for the next lookup's whole backward."""
        g1, f1 = self.fmap1_buffer()
        g2, f2 = self.fmap2_buffer()
        return g1, g2, f1 | f2

    def defer(self, sort_state, records, radius, scale):
        """Keep a lookup's grad_fmap2 records for one pull over many lookups."""
        if self.pull_params not in (None, (radius, scale)):
            self.flush()
        self.pull_params = (radius, scale)
        self.pending.append((sort_state, records))
        if len(self.pending) >= self.MAX_PENDING:
            self.flush()

    def flush(self):
        """grad_fmap2 of the deferred lookups, added into g2 in one pass."""
        if not self.pending:
            return
        radius, scale = self.pull_params
        g2, flag = self.fmap2_buffer()
        pyramid_corr_backward_fmap2_pull(self.fmap1, g2, radius, self.levels, scale,
                                         [p[0] for p in self.pending],
                                         [p[1] for p in self.pending], flag)
        self.pending = []
        self.pull_params = None


class LookupGradSink(torch.autograd.Function):
    """Joins a block's lookups to its NCHW feature maps through one token.

    The token (a 0-dim tensor) is an input of every lookup; its gradient is
    zero, and this backward runs after every lookup's backward (autograd
    waits for all of the token's gradients), returning the accumulated NCHW
    gradients of fmap1 and fmap2.
    """

    @staticmethod
    def forward(ctx, fmap1, fmap2, state):
        ctx.state = state
        ctx.dtype = fmap2.dtype
        return fmap1.new_zeros(())

    @staticmethod
    def backward(ctx, _):
        st = ctx.state
        st.flush()
        g1 = g2 = None
        if st.g1 is not None:
            if ctx.needs_input_grad[0]:
                g1 = nhwc_to_nchw(st.g1)
            if ctx.needs_input_grad[1]:
                g2 = pyramid_build_backward(st.g2, st.fmap2_shape, st.levels, ctx.dtype)
        st.g1 = st.g2 = None
        return g1, g2, None


class PyramidLookup(torch.autograd.Function):
    """One lookup of a pyramid block whose gradients go to ``LookupGrads``."""

    @staticmethod
    def forward(ctx, token, coords, state, radius, levels, scale):
        coords = coords.contiguous()
        # The backward reuses this forward's pixel sort (tensor-core engine).
        nb = sort_state_bytes(state.fmap1, state.fmap2_packed, radius, levels)
        sort_state = (torch.empty(nb, dtype=torch.uint8, device=coords.device)
                      if nb else None)
        corr = pyramid_corr_forward(state.fmap1, state.fmap2_packed, coords, radius, levels,
                                    1, False, scale, sort_state=sort_state)
        ctx.save_for_backward(coords)
        ctx.state = state
        ctx.sort_state = sort_state
        ctx.params = (int(radius), int(levels), float(scale))
        return corr

    @staticmethod
    def backward(ctx, corr_grad):
        (coords,) = ctx.saved_tensors
        st = ctx.state
        radius, levels, scale = ctx.params
        nrec = (records_bytes(st.fmap1, st.fmap2_packed, radius, levels)
                if ctx.sort_state is not None and DEFER_FMAP2 else 0)
        if nrec:
            # grad_fmap1 now; grad_fmap2 with the block's other lookups in
            # one pass when the sink runs (or when MAX_PENDING have gathered)
            g1, flag = st.fmap1_buffer()
            records = torch.empty(nrec, dtype=torch.uint8, device=coords.device)
            pyramid_corr_backward_fmap1(st.fmap1, st.fmap2_packed, coords, corr_grad, radius,
                                        levels, scale, g1, flag, ctx.sort_state, records)
            st.defer(ctx.sort_state, records, radius, scale)
        else:
            g1, g2, flags = st.buffers()
            pyramid_corr_backward(st.fmap1, st.fmap2_packed, coords, corr_grad, radius, levels,
                                  1, False, scale, out=(g1, g2), accumulate=flags,
                                  sort_state=ctx.sort_state)
        ctx.sort_state = None
        gc = torch.zeros_like(coords) if ctx.needs_input_grad[1] else None
        return corr_grad.new_zeros(()), gc, None, None, None, None


class SpatialCorr(torch.autograd.Function):
    """Spatial correlation on NCHW inputs, out [B, RD, RD, H, W]."""

    @staticmethod
    def forward(ctx, in1, in2, radius, dilation, scale):
        in1 = in1.contiguous()
        in2 = in2.contiguous()
        out = spatial_forward(in1, in2, int(radius), int(dilation), float(scale))
        ctx.save_for_backward(in1, in2)
        ctx.params = (int(radius), int(dilation), float(scale))
        return out

    @staticmethod
    def backward(ctx, g):
        in1, in2 = ctx.saved_tensors
        radius, dilation, scale = ctx.params
        g1, g2 = spatial_backward(in1, in2, g, radius, dilation, scale,
                                  ctx.needs_input_grad[0], ctx.needs_input_grad[1])
        return g1, g2, None, None, None


def identity_coords(b, h, w, dtype, device) -> torch.Tensor:
    """Identity grid [B, 2, H, W], channel 0 = x (blocks.py:615-620)."""
    ys = torch.arange(h, device=device, dtype=dtype)
    xs = torch.arange(w, device=device, dtype=dtype)
    gy, gx = torch.meshgrid(ys, xs, indexing="ij")
    return torch.stack([gx, gy], dim=0)[None].repeat(b, 1, 1, 1).contiguous()


def spatial_corr(in1, in2, radius, dilation=1, scale=1.0) -> torch.Tensor:
    """[B, RD, RD, H, W] spatial correlation of NCHW maps, any radius.

    radius <= 4 runs the dedicated shift kernel; larger windows run the
    pyramid engine with one level, y-major order and identity coordinates
    (the route the reference's CUDA sampler always takes, blocks.py:682-694).
    """
    _require_cuda(in1, in2)
    _dtype_code(in1)
    if in2.dtype != in1.dtype:
        raise RuntimeError("input1 and input2 must have the same dtype")
    lc = torch.ops.localcorr
    if radius <= SPATIAL_KERNEL_MAX_RADIUS:
        return lc.spatial_corr(in1, in2, int(radius), int(dilation), float(scale))
    b, c, h, w = in1.shape
    f1 = lc.nchw_to_nhwc(in1)
    f2 = lc.nchw_to_nhwc(in2).reshape(b, -1)
    coords = identity_coords(b, h, w, torch.float32, in1.device)
    corr = lc.pyramid_corr(f1, f2, coords, int(radius), 1, int(dilation), True, float(scale), 0, 0)
    rd = 2 * radius + 1
    return corr.view(b, rd, rd, h, w)


def default_scale(c: int) -> float:
    return 1.0 / math.sqrt(c)
