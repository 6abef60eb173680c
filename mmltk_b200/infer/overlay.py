"""RGBA overlays for the headless live / annotation path.

Reference: the draw kernels of `src/rfdetr/cuda/draw_cuda.cu:207-708` (analysis overlay, composite,
BGR->RGBA copy, manual masks and mask runs, box outline, selection handles, polyline, points,
skeleton, label colours).  The reference shares its overlay with a browser through EGL / DMA-BUF
surfaces; here every overlay is a plain CUDA uint8 [H, W, 4] tensor (RGBA, rows may be pitched)
that a caller composites onto a frame or writes to a file.

CUDA tensors run the sm_100a kernels of ``csrc/kernels/overlay.cu``; CPU tensors run the same
raster rules written with torch ops, which are the tests' oracle:

* a pixel is on a stroke when the distance from its centre to the segment is at most
  thickness / 2 + 0.5 (squared: <= t^2/4 + 1/4);
* a disc of radius r covers pixels whose centre offset (dx, dy) has dx^2 + dy^2 <= r^2;
* a box outline covers the pixels within ``thickness`` of the box edge, inside or outside;
* selection handles are (2r+1)-pixel squares at the four corners and four edge midpoints;
* "over" compositing: c = c + a (s - c), alpha = a_s + a_d (1 - a_s), a = a_s / 255.
"""
from __future__ import annotations

from typing import Optional, Sequence

import torch

from ..ops._ext import kernels

__all__ = ["overlay_detections", "composite_rgba", "copy_rgb_to_rgba", "manual_mask", "manual_mask_runs",
           "box_outline", "selection_handles", "polyline", "points", "skeleton", "label_colors"]


def _rgba(color: Sequence[int]):
    c = [int(v) for v in color]
    return c + [255] if len(c) == 3 else c


def _put(ov: torch.Tensor, sel: torch.Tensor, color) -> None:
    ov[sel] = torch.tensor(_rgba(color), dtype=torch.uint8)


def _grid(h: int, w: int):
    ys, xs = torch.meshgrid(torch.arange(h), torch.arange(w), indexing="ij")
    return xs, ys


def overlay_detections(ov: torch.Tensor, boxes: torch.Tensor, colors: torch.Tensor,
                       masks: Optional[torch.Tensor] = None, thickness: int = 2, mask_alpha: int = 115) -> None:
    """Detections into an RGBA overlay in place: mask pixels in the instance colour at
    ``mask_alpha``, box outlines at full alpha (later instances on top, outlines over masks)."""
    if ov.is_cuda:
        kernels().overlay_detections_(ov, boxes.float().contiguous(), colors.to(torch.uint8).contiguous(),
                                      None if masks is None else masks.to(torch.uint8).contiguous(), thickness,
                                      mask_alpha)
        return
    H, W = ov.shape[:2]
    xs, ys = _grid(H, W)
    hit = torch.full((H, W), -1, dtype=torch.long)
    outline = torch.zeros(H, W, dtype=torch.bool)
    n = boxes.shape[0]
    if masks is not None:
        for i in range(n):
            hit[masks[i].bool()] = i
    t = thickness
    for i in range(n):
        x0, y0, x1, y1 = (float(v) for v in boxes[i])
        inside = (xs >= x0 - t) & (xs <= x1 + t) & (ys >= y0 - t) & (ys <= y1 + t)
        core = (xs > x0 + t - 1) & (xs < x1 - t + 1) & (ys > y0 + t - 1) & (ys < y1 - t + 1)
        e = inside & ~core
        hit[e] = i
        outline |= e
    for i in range(n):
        sel = hit == i
        if sel.any():
            c = colors[i].tolist()
            ov[sel & outline] = torch.tensor(c + [255], dtype=torch.uint8)
            ov[sel & ~outline] = torch.tensor(c + [int(mask_alpha)], dtype=torch.uint8)


def composite_rgba(dst: torch.Tensor, src: torch.Tensor, swap_rb: bool = False) -> None:
    """``src`` RGBA over ``dst`` ([H, W, 3] or [H, W, 4]) in place."""
    if dst.is_cuda:
        kernels().composite_rgba_(dst, src, swap_rb)
        return
    a = src[..., 3:4].float() * (1.0 / 255.0)
    s = src[..., [2, 1, 0]] if swap_rb else src[..., :3]
    d = dst[..., :3].float()
    dst[..., :3] = torch.clamp(d + a * (s.float() - d) + 0.5, max=255.0).to(torch.uint8)
    if dst.shape[-1] == 4:
        dst[..., 3] = torch.clamp(src[..., 3].float() + dst[..., 3].float() * (1 - a[..., 0]) + 0.5,
                                  max=255.0).to(torch.uint8)


def copy_rgb_to_rgba(src: torch.Tensor, swap_rb: bool = False, alpha: int = 255) -> torch.Tensor:
    if src.is_cuda:
        return kernels().copy_rgb_to_rgba(src, swap_rb, alpha)
    rgb = src[..., [2, 1, 0]] if swap_rb else src
    return torch.cat([rgb, torch.full_like(src[..., :1], alpha)], -1)


def manual_mask(ov: torch.Tensor, x0: int, y0: int, mask: torch.Tensor, color) -> None:
    """A binary mask [h, w] painted into the overlay with its top-left corner at (x0, y0)."""
    if ov.is_cuda:
        kernels().manual_mask_(ov, x0, y0, mask.to(torch.uint8).contiguous(), _rgba(color))
        return
    H, W = ov.shape[:2]
    h, w = mask.shape
    ys, xs = torch.nonzero(mask.bool(), as_tuple=True)
    gx, gy = xs + x0, ys + y0
    ok = (gx >= 0) & (gy >= 0) & (gx < W) & (gy < H)
    ov[gy[ok], gx[ok]] = torch.tensor(_rgba(color), dtype=torch.uint8)


def manual_mask_runs(ov: torch.Tensor, x0: int, y0: int, w: int, h: int, runs: torch.Tensor, color) -> None:
    """Run-length mask: ``runs`` [n, 2] (start, length) of row-major indices in a w x h region."""
    if ov.is_cuda:
        kernels().manual_mask_runs_(ov, x0, y0, w, h, runs.to(torch.int32).contiguous(), _rgba(color))
        return
    m = torch.zeros(h * w, dtype=torch.bool)
    for s, n in runs.tolist():
        m[s:min(s + n, h * w)] = True
    manual_mask(ov, x0, y0, m.view(h, w), color)


def box_outline(ov: torch.Tensor, box: Sequence[int], thickness: int, color) -> None:
    if ov.is_cuda:
        kernels().box_outline_(ov, [int(v) for v in box], thickness, _rgba(color))
        return
    H, W = ov.shape[:2]
    xs, ys = _grid(H, W)
    x1, y1, x2, y2 = (int(v) for v in box)
    t = max(1, int(thickness))
    inside = (xs >= x1 - t) & (xs <= x2 + t) & (ys >= y1 - t) & (ys <= y2 + t)
    core = (xs > x1 + t - 1) & (xs < x2 - t + 1) & (ys > y1 + t - 1) & (ys < y2 - t + 1)
    _put(ov, inside & ~core, color)


def selection_handles(ov: torch.Tensor, box: Sequence[int], radius: int, color) -> None:
    if ov.is_cuda:
        kernels().selection_handles_(ov, [int(v) for v in box], radius, _rgba(color))
        return
    H, W = ov.shape[:2]
    xs, ys = _grid(H, W)
    x1, y1, x2, y2 = (int(v) for v in box)
    r = max(1, int(radius))
    mx, my = (x1 + x2) // 2, (y1 + y2) // 2
    sel = torch.zeros(H, W, dtype=torch.bool)
    for hx, hy in ((x1, y1), (mx, y1), (x2, y1), (x2, my), (x2, y2), (mx, y2), (x1, y2), (x1, my)):
        sel |= ((xs - hx).abs() <= r) & ((ys - hy).abs() <= r)
    _put(ov, sel, color)


def _segments_cpu(ov, pts, pairs, thickness, color):
    H, W = ov.shape[:2]
    xs, ys = _grid(H, W)
    xs, ys = xs.float(), ys.float()
    t = max(1, int(thickness))
    lim = 0.25 * t * t + 0.25
    sel = torch.zeros(H, W, dtype=torch.bool)
    for ia, ib in pairs:
        ax, ay = (float(v) for v in pts[ia])
        bx, by = (float(v) for v in pts[ib])
        dx, dy = bx - ax, by - ay
        l2 = dx * dx + dy * dy
        tt = ((xs - ax) * dx + (ys - ay) * dy) / l2 if l2 > 0 else torch.zeros_like(xs)
        tt = tt.clamp(0, 1)
        ex, ey = xs - (ax + tt * dx), ys - (ay + tt * dy)
        sel |= ex * ex + ey * ey <= lim
    _put(ov, sel, color)


def polyline(ov: torch.Tensor, pts: torch.Tensor, closed: bool, thickness: int, color) -> None:
    """Thick polyline through ``pts`` [n, 2] integer (x, y)."""
    if ov.is_cuda:
        kernels().polyline_(ov, pts.to(torch.int32).contiguous(), closed, thickness, _rgba(color))
        return
    n = pts.shape[0]
    if n < 2:
        return
    pairs = [(i, i + 1) for i in range(n - 1)] + ([(n - 1, 0)] if closed else [])
    _segments_cpu(ov, pts, pairs, thickness, color)


def points(ov: torch.Tensor, pts: torch.Tensor, radius: int, color) -> None:
    if ov.is_cuda:
        kernels().points_(ov, pts.to(torch.int32).contiguous(), radius, _rgba(color))
        return
    H, W = ov.shape[:2]
    xs, ys = _grid(H, W)
    r = max(0, int(radius))
    sel = torch.zeros(H, W, dtype=torch.bool)
    for cx, cy in pts.tolist():
        sel |= (xs - cx) ** 2 + (ys - cy) ** 2 <= r * r
    _put(ov, sel, color)


def skeleton(ov: torch.Tensor, pts: torch.Tensor, edges: torch.Tensor, thickness: int, radius: int, color) -> None:
    """Keypoint skeleton: ``edges`` [m, 2] point-index pairs as thick segments, joints as discs."""
    if ov.is_cuda:
        kernels().skeleton_(ov, pts.to(torch.int32).contiguous(), edges.to(torch.int32).contiguous(), thickness,
                            radius, _rgba(color))
        return
    n = pts.shape[0]
    pairs = [(a, b) for a, b in edges.tolist() if 0 <= a < n and 0 <= b < n]
    _segments_cpu(ov, pts, pairs, thickness, color)
    if radius > 0:
        points(ov, pts, radius, color)


def label_colors(labels: torch.Tensor) -> torch.Tensor:
    """[n] class ids -> [n, 3] uint8 RGB: hue = frac(id * 0.618...) on a full-saturation wheel, so
    neighbouring ids get distant colours."""
    if labels.is_cuda:
        return kernels().label_colors(labels.to(torch.int32).contiguous())
    hue = torch.remainder(labels.clamp(min=0).float() * 0.618033988749895, 1.0) * 6.0
    sector = hue.floor()
    f = hue - sector
    q = 1 - f
    one, zero = torch.ones_like(f), torch.zeros_like(f)
    table = [(one, f, zero), (q, one, zero), (zero, one, f), (zero, q, one), (f, zero, one), (one, zero, q)]
    out = torch.zeros(labels.numel(), 3)
    s = sector.long() % 6
    for k, (r, g, b) in enumerate(table):
        m = s == k
        out[m] = torch.stack([r, g, b], -1)[m]
    return (out * 255 + 0.5).to(torch.uint8)
