"""CPU oracle of the localcorr hot path — TEST INFRASTRUCTURE ONLY.

Restates, in plain PyTorch on the CPU (float64 by default), the reference's
algorithm for the pyramid local correlation and the spatial correlation, so
the CUDA engine can be checked against it. Only tests/, __graft_entry__.smoke()
and bench.py's cpu_baseline / reference arm may import this module, and only
as the checker or the timed CPU baseline; the product (localcorr_b200) never
imports it.

Pinned against the reference itself: tests/golden/make_golden.py runs the
reference's own Python implementations (imported from a checkout) on small
seeded cases and stores inputs/outputs/gradients as fixtures;
tests/test_oracle_golden.py checks every function here against them.

Semantics (reference files cited per function):
  * pyramid: 2x2 avg_pool2d chain with floor-halved dims;
  * per level l, coordinate c/2^l, x0 = floor, frac weights
    wa=(1-dx)(1-dy), wb=dx(1-dy), wc=(1-dx)dy, wd=dx*dy, each corner zero
    outside the level map (per-corner masks);
  * taps (iy, ix) at x0 - r*dil + dil*ix, y0 - r*dil + dil*iy;
  * channel d = iy + RD*ix (RAFT order) or ix + RD*iy (ymajor).
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def build_pyramid(fmap2: torch.Tensor, levels: int) -> list[torch.Tensor]:
    """NCHW pyramid by repeated 2x2 average pooling.

    Follows blocks.py:371-373 and onnx_generic.py:95-97.
    """
    pyr = [fmap2]
    for _ in range(1, levels):
        pyr.append(F.avg_pool2d(pyr[-1], 2, stride=2))
    return pyr


def _corner_gather(f2flat: torch.Tensor, xs: torch.Tensor, ys: torch.Tensor, h: int, w: int):
    """f2flat [B, C, h*w]; xs, ys integer [B, P]. Returns [B, C, P] with zeros
    where (ys, xs) is outside the map (the per-corner masks of
    sycl_pyramid/test_kernel.cpp:64-71)."""
    valid = (xs >= 0) & (xs < w) & (ys >= 0) & (ys < h)
    idx = (ys.clamp(0, h - 1) * w + xs.clamp(0, w - 1)).unsqueeze(1)
    idx = idx.expand(-1, f2flat.shape[1], -1)
    vals = torch.gather(f2flat, 2, idx)
    return vals * valid.unsqueeze(1).to(vals.dtype)


def pyramid_corr(fmap1: torch.Tensor, fmap2: torch.Tensor, coords: torch.Tensor, levels: int,
                 radius: int, dilation: int = 1, ymajor: bool = False,
                 dtype: torch.dtype = torch.float64) -> torch.Tensor:
    """Unscaled pyramid local correlation [B, L, RD^2, H, W], tap by tap.

    fmap1/fmap2 NCHW, coords [B, 2, H, W] (x, y; level-0 pixels). Follows
    the double-precision CPU reference of the reference kernel
    (sycl_pyramid/test_kernel.cpp:26-91) and the per-displacement reference
    (tests/_reference.py:43-75), vectorised over pixels. Differentiable with
    respect to fmap1 and fmap2 (through the pooling chain).
    """
    f1 = fmap1.to(dtype)
    f2 = fmap2.to(dtype)
    co = coords.to(dtype)
    b, c, h, w = f1.shape
    rd = 2 * radius + 1
    p = h * w
    f1flat = f1.reshape(b, c, p)
    out_levels = []
    for lvl, f2l in enumerate(build_pyramid(f2, levels)):
        hl, wl = f2l.shape[-2:]
        f2flat = f2l.reshape(b, c, hl * wl)
        clx = co[:, 0].reshape(b, p) / float(2 ** lvl)
        cly = co[:, 1].reshape(b, p) / float(2 ** lvl)
        x0f = torch.floor(clx)
        y0f = torch.floor(cly)
        dx = clx - x0f
        dy = cly - y0f
        xb = x0f.long() - radius * dilation
        yb = y0f.long() - radius * dilation
        wa = ((1 - dx) * (1 - dy)).unsqueeze(1)
        wb = (dx * (1 - dy)).unsqueeze(1)
        wc = ((1 - dx) * dy).unsqueeze(1)
        wd = (dx * dy).unsqueeze(1)
        planes = [None] * (rd * rd)
        for iy in range(rd):
            y0 = yb + dilation * iy
            for ix in range(rd):
                x0 = xb + dilation * ix
                f2v = (wa * _corner_gather(f2flat, x0, y0, hl, wl)
                       + wb * _corner_gather(f2flat, x0 + 1, y0, hl, wl)
                       + wc * _corner_gather(f2flat, x0, y0 + 1, hl, wl)
                       + wd * _corner_gather(f2flat, x0 + 1, y0 + 1, hl, wl))
                d = ix + rd * iy if ymajor else iy + rd * ix
                planes[d] = (f1flat * f2v).sum(dim=1)
        out_levels.append(torch.stack(planes, dim=1).reshape(b, rd * rd, h, w))
    return torch.stack(out_levels, dim=1)


def pyramid_corr_points(fmap1: torch.Tensor, fmap2: torch.Tensor, coords: torch.Tensor,
                        levels: int, radius: int, points: torch.Tensor,
                        dilation: int = 1, ymajor: bool = False) -> torch.Tensor:
    """pyramid_corr restricted to a pixel subset (float64).

    points: int64 [N, 3] rows (b, h, w). Returns [N, L, RD^2]. Used for spot
    checks at full benchmark sizes, where the dense oracle is too slow.
    """
    f1 = fmap1.double()
    co = coords.double()
    rd = 2 * radius + 1
    bi, hi, wi = points[:, 0], points[:, 1], points[:, 2]
    f1p = f1[bi, :, hi, wi]  # [N, C]
    cx = co[bi, 0, hi, wi]
    cy = co[bi, 1, hi, wi]
    res = []
    for lvl, f2l in enumerate(build_pyramid(fmap2.double(), levels)):
        hl, wl = f2l.shape[-2:]
        clx, cly = cx / float(2 ** lvl), cy / float(2 ** lvl)
        x0f, y0f = torch.floor(clx), torch.floor(cly)
        dx, dy = clx - x0f, cly - y0f
        xb = x0f.long() - radius * dilation
        yb = y0f.long() - radius * dilation
        wts = [((1 - dx) * (1 - dy)), (dx * (1 - dy)), ((1 - dx) * dy), (dx * dy)]
        out = torch.zeros(len(points), rd * rd, dtype=torch.float64)
        for iy in range(rd):
            for ix in range(rd):
                x0 = xb + dilation * ix
                y0 = yb + dilation * iy
                acc = torch.zeros_like(f1p)
                for k, (ox, oy) in enumerate(((0, 0), (1, 0), (0, 1), (1, 1))):
                    xx, yy = x0 + ox, y0 + oy
                    valid = (xx >= 0) & (xx < wl) & (yy >= 0) & (yy < hl)
                    v = f2l[bi, :, yy.clamp(0, hl - 1), xx.clamp(0, wl - 1)]
                    acc = acc + (wts[k] * valid.double()).unsqueeze(1) * v
                d = ix + rd * iy if ymajor else iy + rd * ix
                out[:, d] = (f1p * acc).sum(dim=1)
        res.append(out)
    return torch.stack(res, dim=1)


def _tap_setup(co, bi, hi, wi, lvl, radius):
    """Level-lvl window base and bilinear weights of the pixels (bi, hi, wi)."""
    cx = co[bi, 0, hi, wi] / float(2 ** lvl)
    cy = co[bi, 1, hi, wi] / float(2 ** lvl)
    x0f, y0f = torch.floor(cx), torch.floor(cy)
    dx, dy = cx - x0f, cy - y0f
    wts = [(1 - dx) * (1 - dy), dx * (1 - dy), (1 - dx) * dy, dx * dy]
    return x0f.long() - radius, y0f.long() - radius, wts


_CORNERS = ((0, 0), (1, 0), (0, 1), (1, 1))


def pyramid_corr_points_grad_fmap1(fmap1: torch.Tensor, fmap2: torch.Tensor,
                                   coords: torch.Tensor, levels: int, radius: int,
                                   points: torch.Tensor, grad_out: torch.Tensor,
                                   ymajor: bool = False) -> torch.Tensor:
    """Gradient of sum(grad_out * pyramid_corr) w.r.t. fmap1 at a pixel subset.

    points: int64 [N, 3] rows (b, h, w); grad_out [B, L, RD^2, H, W]
    (unscaled: multiply by the output scale outside). Returns [N, C] float64:
      gf1[p, c] = sum_l sum_(iy,ix) g[p, l, d] * bilinear(f2_l, tap)[c]
    with the per-corner masks, as the reference backward accumulates its
    fmap1 row (cuda_pyramid/localcorr_cuda_pyramid_kernel.cu:870-899).
    Dilation 1 (the tensor-core engine's configuration)."""
    go = grad_out.double()
    co = coords.double()
    rd = 2 * radius + 1
    bi, hi, wi = points[:, 0], points[:, 1], points[:, 2]
    n, c = len(points), fmap1.shape[1]
    acc = torch.zeros(n, c, dtype=torch.float64)
    for lvl, f2l in enumerate(build_pyramid(fmap2.double(), levels)):
        hl, wl = f2l.shape[-2:]
        xb, yb, wts = _tap_setup(co, bi, hi, wi, lvl, radius)
        for iy in range(rd):
            for ix in range(rd):
                d = ix + rd * iy if ymajor else iy + rd * ix
                g = go[bi, lvl, d, hi, wi]
                for k, (ox, oy) in enumerate(_CORNERS):
                    xx, yy = xb + ix + ox, yb + iy + oy
                    valid = (xx >= 0) & (xx < wl) & (yy >= 0) & (yy < hl)
                    v = f2l[bi, :, yy.clamp(0, hl - 1), xx.clamp(0, wl - 1)]
                    acc += (g * wts[k] * valid.double()).unsqueeze(1) * v
    return acc


def pyramid_corr_points_grad_levels(fmap1: torch.Tensor, fmap2: torch.Tensor,
                                    coords: torch.Tensor, levels: int, radius: int,
                                    positions: torch.Tensor, grad_out: torch.Tensor,
                                    ymajor: bool = False) -> torch.Tensor:
    """Gradient of sum(grad_out * pyramid_corr) w.r.t. the pyramid levels at
    a subset of level positions (the packed float32 gradient the C ABI
    backward writes, before the pyramid build's own gradient).

    positions: int64 [N, 4] rows (b, l, y, x) with (y, x) inside level l.
    Returns [N, C] float64: the sum over every pixel p of image b and every
    tap/corner of p's level-l window that lands on (y, x) of
      g[p, l, d] * w_corner(p) * fmap1[p]
    which is the reference backward's atomic scatter
    (cuda_pyramid/localcorr_cuda_pyramid_kernel.cu:901-913) gathered at one
    target. Dilation 1."""
    go = grad_out.double()
    co = coords.double()
    f1 = fmap1.double()
    b_all, c, h, w = f1.shape
    rd = 2 * radius + 1
    out = torch.zeros(len(positions), c, dtype=torch.float64)
    for i, (b, lvl, y, x) in enumerate(positions.tolist()):
        cx = co[b, 0] / float(2 ** lvl)
        cy = co[b, 1] / float(2 ** lvl)
        x0f, y0f = torch.floor(cx), torch.floor(cy)
        dx, dy = cx - x0f, cy - y0f
        xb = x0f.long() - radius
        yb = y0f.long() - radius
        # pixels whose window (grid rows/cols base .. base + rd) holds (y, x)
        near = (x >= xb) & (x <= xb + rd) & (y >= yb) & (y <= yb + rd)
        hs, ws = torch.nonzero(near, as_tuple=True)
        if len(hs) == 0:
            continue
        wts = [(1 - dx) * (1 - dy), dx * (1 - dy), (1 - dx) * dy, dx * dy]
        coef = torch.zeros(len(hs), dtype=torch.float64)
        for k, (ox, oy) in enumerate(_CORNERS):
            ix = x - ox - xb[hs, ws]
            iy = y - oy - yb[hs, ws]
            ok = (ix >= 0) & (ix < rd) & (iy >= 0) & (iy < rd)
            ixc, iyc = ix.clamp(0, rd - 1), iy.clamp(0, rd - 1)
            d = ixc + rd * iyc if ymajor else iyc + rd * ixc
            g = go[b, lvl][d, hs, ws]
            coef += g * wts[k][hs, ws] * ok.double()
        out[i] = (coef.unsqueeze(1) * f1[b, :, hs, ws].T).sum(dim=0)
    return out


def _pixel_to_grid(coords: torch.Tensor, size: int) -> torch.Tensor:
    """Pixel coordinate -> grid_sample coordinate with align_corners=False
    (onnx_generic.py:34-42)."""
    return (coords + 0.5) / size * 2.0 - 1.0


def pyramid_corr_matmul(fmap1: torch.Tensor, fmap2: torch.Tensor, coords: torch.Tensor,
                        levels: int, radius: int, tile_rows: int = 8) -> torch.Tensor:
    """The reference's CPU formulation (onnx_generic.py:58-156), restated.

    Per level and per band of fmap1 rows, the all-pairs tile
    M[p, q] = <fmap1[p], fmap2_l[q]> is one matmul, and the (2r+1)^2 taps
    of every pixel are bilinear samples of its row of M (grid_sample,
    align_corners=False, zero padding), laid out so the channel is
    ix*rd + iy. Computes in fmap1's dtype; this is the timed CPU baseline.
    """
    b, c, h, w = fmap1.shape
    rd = 2 * radius + 1
    axis = torch.arange(rd, dtype=torch.float32) - radius
    f1 = fmap1.reshape(b, c, -1).permute(0, 2, 1)  # [B, P, C]
    outs = []
    for lvl, f2l in enumerate(build_pyramid(fmap2, levels)):
        hl, wl = f2l.shape[-2:]
        f2 = f2l.reshape(b, c, -1)  # [B, C, Q]
        cl = coords.to(torch.float32) / float(2 ** lvl)
        gx = _pixel_to_grid(cl[:, 0], wl)
        gy = _pixel_to_grid(cl[:, 1], hl)
        dxn = (axis * 2.0 / wl).view(1, 1, 1, rd, 1)
        dyn = (axis * 2.0 / hl).view(1, 1, 1, 1, rd)
        tiles = []
        for r0 in range(0, h, tile_rows):
            r1 = min(h, r0 + tile_rows)
            pt = (r1 - r0) * w
            grid_x = (gx[:, r0:r1, :, None, None] + dxn).expand(b, r1 - r0, w, rd, rd)
            grid_y = (gy[:, r0:r1, :, None, None] + dyn).expand(b, r1 - r0, w, rd, rd)
            grid = torch.stack([grid_x, grid_y], dim=-1).reshape(b * pt, rd, rd, 2)
            m = torch.matmul(f1[:, r0 * w:r1 * w], f2).reshape(b * pt, 1, hl, wl)
            s = F.grid_sample(m, grid.to(m.dtype), mode="bilinear", padding_mode="zeros",
                              align_corners=False)
            tiles.append(s.reshape(b, pt, rd * rd))
        corr = torch.cat(tiles, dim=1).reshape(b, h, w, rd * rd).permute(0, 3, 1, 2)
        outs.append(corr)
    return torch.stack(outs, dim=1)


def spatial_corr(in1: torch.Tensor, in2: torch.Tensor, radius: int, dilation: int = 1,
                 dtype: torch.dtype = torch.float64) -> torch.Tensor:
    """[B, RD, RD, H, W] spatial correlation by shifted slices, zero padded.

    out[b, iy, ix, h, w] = sum_c in1[b,c,h,w] * in2[b,c,h+dil*(iy-r),w+dil*(ix-r)].
    Follows tests/_reference.py:78-125 and onnx_generic.py:159-198.
    """
    x1 = in1.to(dtype)
    x2 = in2.to(dtype)
    b, c, h, w = x1.shape
    rd = 2 * radius + 1
    pad = radius * dilation
    x2p = F.pad(x2, (pad, pad, pad, pad))
    rows = []
    for iy in range(rd):
        cols = []
        for ix in range(rd):
            y0 = iy * dilation
            x0 = ix * dilation
            cols.append((x1 * x2p[:, :, y0:y0 + h, x0:x0 + w]).sum(dim=1))
        rows.append(torch.stack(cols, dim=1))
    return torch.stack(rows, dim=1)


def block_forward(fmap1, fmap2, coords, levels, radius, dtype=torch.float64):
    """What the RAFT block returns: [B, L*RD^2, H, W] divided by sqrt(C)
    (blocks.py:391-411)."""
    b, c, h, w = fmap1.shape
    out = pyramid_corr(fmap1, fmap2, coords, levels, radius, dtype=dtype)
    return out.reshape(b, -1, h, w) / math.sqrt(c)


def block_grads(fmap1, fmap2, coords, levels, radius, grad_out, dtype=torch.float64):
    """(out, grad_fmap1, grad_fmap2) of the RAFT block under upstream grad_out."""
    f1 = fmap1.detach().to(dtype).requires_grad_(True)
    f2 = fmap2.detach().to(dtype).requires_grad_(True)
    out = block_forward(f1, f2, coords.to(dtype), levels, radius, dtype=dtype)
    g1, g2 = torch.autograd.grad(out, [f1, f2], grad_out.to(dtype).reshape(out.shape))
    return out.detach(), g1, g2


def spatial_grads(in1, in2, radius, grad_out, dilation=1, dtype=torch.float64):
    x1 = in1.detach().to(dtype).requires_grad_(True)
    x2 = in2.detach().to(dtype).requires_grad_(True)
    out = spatial_corr(x1, x2, radius, dilation, dtype=dtype)
    g1, g2 = torch.autograd.grad(out, [x1, x2], grad_out.to(dtype).reshape(out.shape))
    return out.detach(), g1, g2


# ---- seeded synthetic inputs (shapes and distributions of the benchmark
# configurations; tests/_reference.py:14-35 for the small-case generators) ----

def make_fmaps(batch, channels, height, width, seed=0, dist="normal"):
    g = torch.Generator().manual_seed(seed)
    if dist == "uniform":
        f1 = torch.rand(batch, channels, height, width, generator=g) * 2 - 1
        f2 = torch.rand(batch, channels, height, width, generator=g) * 2 - 1
    else:
        f1 = torch.randn(batch, channels, height, width, generator=g)
        f2 = torch.randn(batch, channels, height, width, generator=g)
    return f1, f2


def identity_grid(batch, height, width):
    ys, xs = torch.meshgrid(torch.arange(height, dtype=torch.float32),
                            torch.arange(width, dtype=torch.float32), indexing="ij")
    return torch.stack([xs, ys], dim=0)[None].repeat(batch, 1, 1, 1)


def make_coords_uniform(batch, height, width, max_disp, seed=1):
    """identity + U(-max_disp, max_disp) flow (tests/_reference.py:23-35)."""
    g = torch.Generator().manual_seed(seed)
    flow = torch.rand(batch, 2, height, width, generator=g) * 2 - 1
    return identity_grid(batch, height, width) + flow * max_disp


def make_coords_gauss_oob(batch, height, width, sigma=6.0, oob_frac=0.05, seed=1):
    """identity + N(0, sigma^2) flow with a fraction of pixels pushed out of
    bounds by (W or H) * U(1, 2) (benchmark configuration 2)."""
    g = torch.Generator().manual_seed(seed)
    coords = identity_grid(batch, height, width) + sigma * torch.randn(
        batch, 2, height, width, generator=g)
    pick = torch.rand(batch, height, width, generator=g) < oob_frac
    axis = torch.rand(batch, height, width, generator=g) < 0.5
    sign = torch.where(torch.rand(batch, height, width, generator=g) < 0.5, -1.0, 1.0)
    mag = 1.0 + torch.rand(batch, height, width, generator=g)
    push_x = pick & axis
    push_y = pick & ~axis
    coords[:, 0] += torch.where(push_x, sign * mag * width, torch.zeros(()))
    coords[:, 1] += torch.where(push_y, sign * mag * height, torch.zeros(()))
    return coords


def make_coords_smooth(batch, height, width, amplitude=40.0, seed=1):
    """identity + sum of 4 random sinusoids per axis, |flow| <= amplitude
    (benchmark configuration 4)."""
    g = torch.Generator().manual_seed(seed)
    grid = identity_grid(batch, height, width)
    ys, xs = grid[:, 1], grid[:, 0]
    flow = torch.zeros(batch, 2, height, width)
    for axis in range(2):
        for _ in range(4):
            fx, fy = (torch.rand(2, generator=g) * 2 - 1) * (2 * math.pi / 64)
            ph = torch.rand(1, generator=g) * 2 * math.pi
            amp = torch.rand(1, generator=g) * amplitude / 4
            flow[:, axis] += amp * torch.sin(fx * xs + fy * ys + ph)
    return grid + flow
