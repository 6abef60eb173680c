"""Detection drawing and frame pre-processing on the device.

``draw_detections`` burns masks (alpha blend), box outlines and label bars
(class name + score, built-in 5x7 font) into an 8-bit 3-channel image; on CUDA
this is one kernel (``csrc/kernels/imaging.cu``), on CPU the torch statement
below (boxes, masks and label bars; text glyphs are drawn only on the device).
Reference: the draw kernels of `src/rfdetr/cuda/draw_cuda.cu:64-708` and the
eval sample image written during training.

``letterbox`` maps a camera / file frame to the model input (scale to fit,
centred, grey padding) -- fused with the ImageNet normalisation on CUDA.
"""
from __future__ import annotations

from typing import Dict, List, Optional, Sequence

import torch

from ..ops._ext import kernels

__all__ = ["draw_detections", "draw_reference", "palette", "letterbox", "letterbox_reference", "letterbox_geometry"]


def palette(labels: torch.Tensor) -> torch.Tensor:
    """Stable, well-spread colours per class id: [n, 3] uint8."""
    lab = labels.to(torch.int64).cpu()
    h = (lab * 0.61803398875) % 1.0
    # HSV (h, 0.75, 0.95) -> RGB
    i = (h * 6).floor()
    f = h * 6 - i
    v, s = 0.95, 0.75
    p, q, t = v * (1 - s), v * (1 - s * f), v * (1 - s * (1 - f))
    i = i.long() % 6
    r = torch.stack([torch.full_like(f, v), q, torch.full_like(f, p), torch.full_like(f, p), t, torch.full_like(f, v)], -1)
    g = torch.stack([t, torch.full_like(f, v), torch.full_like(f, v), q, torch.full_like(f, p), torch.full_like(f, p)], -1)
    b = torch.stack([torch.full_like(f, p), torch.full_like(f, p), t, torch.full_like(f, v), torch.full_like(f, v), q], -1)
    rgb = torch.stack([r.gather(-1, i[:, None])[:, 0], g.gather(-1, i[:, None])[:, 0], b.gather(-1, i[:, None])[:, 0]],
                      -1)
    return (rgb * 255).round().to(torch.uint8)


def _labels_text(labels, scores, class_names: Sequence[str], width: int = 24) -> torch.Tensor:
    rows = []
    for l, s in zip(labels.tolist(), scores.tolist()):
        name = class_names[l] if 0 <= l < len(class_names) and class_names[l] else str(l)
        t = f"{name} {100 * s:.0f}%"[:width]
        rows.append(list(t.encode("ascii", "replace")) + [0] * (width - len(t)))
    return torch.tensor(rows, dtype=torch.int8) if rows else torch.zeros(0, width, dtype=torch.int8)


def draw_reference(img: torch.Tensor, boxes: torch.Tensor, colors: torch.Tensor,
                   masks: Optional[torch.Tensor] = None, thickness: int = 2, mask_alpha: float = 0.45) -> torch.Tensor:
    """CPU statement: [H, W, 3] uint8 -> new image with masks and box outlines."""
    out = img.float().clone()
    H, W, _ = out.shape
    ys, xs = torch.meshgrid(torch.arange(H), torch.arange(W), indexing="ij")
    if masks is not None:
        for i in range(boxes.shape[0]):
            m = masks[i].bool()
            out[m] += mask_alpha * (colors[i].float() - out[m])
    for i in range(boxes.shape[0]):
        x0, y0, x1, y1 = boxes[i].tolist()
        inside = (xs >= x0 - thickness) & (xs <= x1 + thickness) & (ys >= y0 - thickness) & (ys <= y1 + thickness)
        core = (xs > x0 + thickness - 1) & (xs < x1 - thickness + 1) & (ys > y0 + thickness - 1) & \
            (ys < y1 - thickness + 1)
        out[inside & ~core] = colors[i].float()
    return (out + 0.5).clamp(0, 255).to(torch.uint8)


def draw_detections(img: torch.Tensor, result: Dict[str, torch.Tensor], class_names: Sequence[str] = (),
                    threshold: float = 0.5, thickness: int = 2, mask_alpha: float = 0.45, text: bool = True,
                    bgr: bool = False) -> torch.Tensor:
    """img [H, W, 3] uint8 (drawn in place on CUDA); result: one image's scores/labels/boxes[/masks]."""
    keep = result["scores"] >= threshold
    boxes = result["boxes"][keep].float()
    labels = result["labels"][keep]
    scores = result["scores"][keep]
    colors = palette(labels)
    if bgr:
        colors = colors.flip(-1)
    masks = result["masks"][keep] if "masks" in result and result["masks"] is not None else None
    if img.is_cuda:
        txt = _labels_text(labels, scores, class_names) if text else None
        kernels().draw_(img, boxes, colors, None if masks is None else masks.to(torch.uint8), txt, thickness,
                        mask_alpha, 2)
        return img
    return draw_reference(img, boxes.cpu(), colors, None if masks is None else masks.cpu(), thickness, mask_alpha)


def letterbox_geometry(src_hw, dst_hw):
    """(scale, tx, ty): dst = src * scale + t (centred, aspect preserved)."""
    sh, sw = src_hw
    dh, dw = dst_hw
    s = min(dw / sw, dh / sh)
    return s, 0.5 * (dw - s * sw), 0.5 * (dh - s * sh)


def letterbox_reference(frame: torch.Tensor, h: int, w: int, bgr: bool = True) -> torch.Tensor:
    """CPU statement of the letterbox kernel: [H, W, 3] uint8 -> [3, h, w] fp32 in [0, 1]."""
    sh, sw = frame.shape[:2]
    s, tx, ty = letterbox_geometry((sh, sw), (h, w))
    ys, xs = torch.meshgrid(torch.arange(h, dtype=torch.float32), torch.arange(w, dtype=torch.float32), indexing="ij")
    sx = (xs + 0.5 - tx) / s - 0.5
    sy = (ys + 0.5 - ty) / s - 0.5
    inside = (sx > -0.5) & (sy > -0.5) & (sx < sw - 0.5) & (sy < sh - 0.5)
    fx = sx.clamp(0, sw - 1)
    fy = sy.clamp(0, sh - 1)
    x0, y0 = fx.long(), fy.long()
    x1, y1 = (x0 + 1).clamp(max=sw - 1), (y0 + 1).clamp(max=sh - 1)
    ax, ay = (fx - x0)[..., None], (fy - y0)[..., None]
    f = frame.float()
    top = f[y0, x0] + ax * (f[y0, x1] - f[y0, x0])
    bot = f[y1, x0] + ax * (f[y1, x1] - f[y1, x0])
    v = top + ay * (bot - top)
    v = torch.where(inside[..., None], v, torch.full_like(v, 128.0))
    if bgr:
        v = v.flip(-1)
    return (v / 255.0).permute(2, 0, 1).contiguous()


def letterbox(frame: torch.Tensor, h: int, w: int, bgr: bool = True, normalize_bf16: bool = True) -> torch.Tensor:
    """[H, W, 3] uint8 frame -> [3, h, w] model input (normalised bf16) or [0,1] fp32."""
    if frame.is_cuda:
        return kernels().letterbox(frame, h, w, bgr, normalize_bf16)
    x = letterbox_reference(frame, h, w, bgr)
    if normalize_bf16:
        mean = torch.tensor([0.485, 0.456, 0.406]).view(3, 1, 1)
        std = torch.tensor([0.229, 0.224, 0.225]).view(3, 1, 1)
        return ((x - mean) / std).to(torch.bfloat16)
    return x
