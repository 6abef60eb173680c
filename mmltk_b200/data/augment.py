"""Fused GPU training augmentation (geometry, resize, colour, noise, blur,
occlusion, single-instance copy-paste) and ImageNet normalisation.

Reference behaviour: `src/rfdetr/gpu_augment.cpp:29-544`,
`src/rfdetr/cuda/gpu_augment_cuda.cu:138-616`, the target side in
`src/rfdetr/target_builder.cpp:338-615`, config defaults in
`include/mmltk/rfdetr/train_types.h:19-42` and the CLI flags in
`src/rfdetr/cli/workflow_cli_shared.h:276-302`.

Split of the work:

* host (C++, ``csrc/host/augment.cpp``): every random draw of the batch, into a
  64-float record per image, plus the augmented padded targets (boxes pushed
  through the forward affine, degenerate or fully covered instances dropped,
  the pasted instance appended) and the donor-cache bookkeeping;
* device (``csrc/kernels/augment.cu``): one fused pass per batch from the
  loader's uint8 pixels to normalised bf16 model input, and one pass that warps
  the target masks with the same records.

:func:`augment_reference` restates the kernel in plain torch (fp32) -- the
CPU path and the oracle of the kernel tests.
"""
from __future__ import annotations

import json
import os

from typing import List, Optional, Sequence, Tuple

import torch

from ..config.train_options import AugGroup as AugmentGroup
from ..config.train_options import AugmentationConfig as AugmentConfig
from ..criterion.targets import Targets
from ..ops._ext import kernels, native

__all__ = ["AugmentGroup", "AugmentConfig", "config_to_native", "GpuAugmenter", "augment_reference", "normalize_images",
           "IMAGENET_MEAN", "IMAGENET_STD", "REC"]

_GROUPS = ("geometry", "resize", "color", "noise", "blur", "occlusion")
IMAGENET_MEAN = (0.485, 0.456, 0.406)
IMAGENET_STD = (0.229, 0.224, 0.225)

# record offsets (csrc/host/augment.h)
_TRACE_FILE = os.environ.get("MMLTK_AUGMENT_TRACE_FILE", "")

REC = dict(inv=0, fwd=6, color=12, color_off=21, noise_mode=24, noise_str=25, blur=26, occ_mode=27, occ_str=28,
           occ_chan=29, erase=30, area_scale=34, flags=35, paste_slot=36, paste_mode=37, paste_inv=38, noise_key=44,
           paste_box=45, floats=64)


def config_to_native(cfg: AugmentConfig) -> dict:
    if not cfg.valid():
        raise ValueError("augmentation: every group needs 0 <= probability <= 1 and "
                         "0 <= min_strength <= max_strength <= 1, and copy-paste probability in [0, 1]")
    d = {g: (getattr(cfg, g).probability, getattr(cfg, g).min_strength, getattr(cfg, g).max_strength)
         for g in _GROUPS}
    d["enabled"] = bool(cfg.enabled)
    d["copy_paste"] = float(cfg.copy_paste_probability)
    return d


def _copy_paste_on(cfg: AugmentConfig) -> bool:
    return cfg.enabled and cfg.copy_paste_probability > 0


# ------------------------------------------------------------------ torch restatement (CPU path / oracle)

_M32 = 0xFFFFFFFF


def _hash32(x: torch.Tensor) -> torch.Tensor:
    x = x & _M32
    x = x ^ (x >> 16)
    x = (x * 0x7FEB352D) & _M32
    x = x ^ (x >> 15)
    x = (x * 0x846CA68B) & _M32
    return x ^ (x >> 16)


def _uniform(key: int, counter: torch.Tensor) -> torch.Tensor:
    h = _hash32(torch.full_like(counter, key) ^ _hash32(counter + 0x68E31DA4))
    return (h >> 8).float() * (1.0 / 16777216.0)


def _sample(plane: torch.Tensor, sx: torch.Tensor, sy: torch.Tensor, blur: float, fill: float) -> torch.Tensor:
    H, W = plane.shape
    fx = (sx * W - 0.5).clamp(0, W - 1)
    fy = (sy * H - 0.5).clamp(0, H - 1)
    x0 = fx.long()
    y0 = fy.long()
    x1 = (x0 + 1).clamp(max=W - 1)
    y1 = (y0 + 1).clamp(max=H - 1)
    ax, ay = fx - x0, fy - y0
    v00, v01, v10, v11 = plane[y0, x0], plane[y0, x1], plane[y1, x0], plane[y1, x1]
    top = v00 + ax * (v01 - v00)
    bot = v10 + ax * (v11 - v10)
    bil = top + ay * (bot - top)
    box = 0.25 * (v00 + v01 + v10 + v11)
    out = bil + blur * (box - bil)
    inside = (sx >= 0) & (sx <= 1) & (sy >= 0) & (sy <= 1)
    return torch.where(inside, out, torch.full_like(out, fill))


def _mask_at(m: torch.Tensor, sx: torch.Tensor, sy: torch.Tensor) -> torch.Tensor:
    H, W = m.shape
    x = torch.round(sx * W - 0.5).long().clamp(0, W - 1)
    y = torch.round(sy * H - 0.5).long().clamp(0, H - 1)
    inside = (sx >= 0) & (sx <= 1) & (sy >= 0) & (sy <= 1)
    return inside & (m[y, x] != 0)


def augment_reference(images: torch.Tensor, records: Optional[torch.Tensor] = None,
                      donors: Optional[torch.Tensor] = None, donor_masks: Optional[torch.Tensor] = None) -> torch.Tensor:
    """images [B,3,H,W] uint8 or float in [0,1]; records [B,64] -> normalised fp32 [B,3,H,W]."""
    x = images.float() / 255 if images.dtype == torch.uint8 else images.float()
    if donors is not None and donors.dtype == torch.uint8:
        donors = donors.float() / 255
    B, _, H, W = x.shape
    mean = torch.tensor(IMAGENET_MEAN).view(3, 1, 1)
    std = torch.tensor(IMAGENET_STD).view(3, 1, 1)
    if records is None:
        return (x.clamp(0, 1) - mean) / std
    rec = records.float().cpu()
    ys, xs = torch.meshgrid(torch.arange(H), torch.arange(W), indexing="ij")
    nx = (xs.float() + 0.5) / W
    ny = (ys.float() + 0.5) / H
    out = torch.empty(B, 3, H, W)
    for b in range(B):
        R = rec[b]
        v = [x[b, c].clone() for c in range(3)]
        if R[REC["flags"]] != 0:
            i = R[REC["inv"]:REC["inv"] + 6]
            sx = i[0] * nx + i[1] * ny + i[2]
            sy = i[3] * nx + i[4] * ny + i[5]
            blur = float(R[REC["blur"]])
            v = [_sample(x[b, c], sx, sy, blur, IMAGENET_MEAN[c]) for c in range(3)]
            slot = int(R[REC["paste_slot"]])
            if slot >= 0 and donors is not None:
                p = R[REC["paste_inv"]:REC["paste_inv"] + 6]
                dx = p[0] * nx + p[1] * ny + p[2]
                dy = p[3] * nx + p[4] * ny + p[5]
                if int(R[REC["paste_mode"]]) == 1:
                    sel = _mask_at(donor_masks[slot].cpu(), dx, dy)
                else:
                    bx = R[REC["paste_box"]:REC["paste_box"] + 4]
                    sel = (dx >= bx[0]) & (dx <= bx[2]) & (dy >= bx[1]) & (dy <= bx[3])
                d = donors[slot].float().cpu()
                v = [torch.where(sel, _sample(d[c], dx, dy, blur, IMAGENET_MEAN[c]), v[c]) for c in range(3)]
        r, g, bl = v
        cm = R[REC["color"]:REC["color"] + 9]
        co = R[REC["color_off"]:REC["color_off"] + 3]
        r, g, bl = (cm[0] * r + cm[1] * g + cm[2] * bl + co[0], cm[3] * r + cm[4] * g + cm[5] * bl + co[1],
                    cm[6] * r + cm[7] * g + cm[8] * bl + co[2])
        key = int(R[REC["noise_key"]:REC["noise_key"] + 1].view(torch.int32).item()) & _M32
        ctr = (ys * W + xs).long() * 16
        mode = int(R[REC["noise_mode"]])
        if mode == 1:
            sig = 0.06 * float(R[REC["noise_str"]])
            n = [sum(_uniform(key, ctr + 4 * c + j) for j in range(4)) - 2.0 for c in range(3)]
            r, g, bl = r + sig * n[0], g + sig * n[1], bl + sig * n[2]
        elif mode == 2:
            salt = _uniform(key, ctr + 12) < 0.02 * float(R[REC["noise_str"]])
            r, g, bl = [torch.where(salt, torch.ones_like(t), t) for t in (r, g, bl)]
        occ = int(R[REC["occ_mode"]])
        ost = float(R[REC["occ_str"]])
        erase = torch.zeros(H, W, dtype=torch.bool)
        if occ == 2:
            erase = _uniform(key, ctr + 13) < 0.05 * ost
        elif occ == 3:
            e = R[REC["erase"]:REC["erase"] + 4]
            erase = (nx >= e[0]) & (nx < e[2]) & (ny >= e[1]) & (ny < e[3])
        ch = [r, g, bl]
        if occ == 1:
            c = int(R[REC["occ_chan"]])
            ch[c] = ch[c] + ost * (IMAGENET_MEAN[c] - ch[c])
        ch = [torch.where(erase, torch.full_like(ch[c], IMAGENET_MEAN[c]), ch[c]) for c in range(3)]
        for c in range(3):
            out[b, c] = (ch[c].clamp(0, 1) - IMAGENET_MEAN[c]) / IMAGENET_STD[c]
    return out


def warp_masks_reference(src: torch.Tensor, donor_masks: Optional[torch.Tensor], rows: torch.Tensor,
                         records: torch.Tensor) -> torch.Tensor:
    """Restatement of the mask warp kernel: rows [N,2] = (image, source row | -(slot+2))."""
    N = rows.shape[0]
    H, W = src.shape[-2:] if src.numel() else donor_masks.shape[-2:]
    ys, xs = torch.meshgrid(torch.arange(H), torch.arange(W), indexing="ij")
    nx = (xs.float() + 0.5) / W
    ny = (ys.float() + 0.5) / H
    out = torch.zeros(N, H, W, dtype=torch.uint8)
    rec = records.float().cpu()
    for n in range(N):
        b, s = int(rows[n, 0]), int(rows[n, 1])
        R = rec[b]
        p = R[REC["paste_inv"]:REC["paste_inv"] + 6]
        dx = p[0] * nx + p[1] * ny + p[2]
        dy = p[3] * nx + p[4] * ny + p[5]
        slot = int(R[REC["paste_slot"]])
        if s >= 0:
            i = R[REC["inv"]:REC["inv"] + 6]
            v = _mask_at(src[s].cpu(), i[0] * nx + i[1] * ny + i[2], i[3] * nx + i[4] * ny + i[5])
            if slot >= 0:
                if int(R[REC["paste_mode"]]) == 1:
                    v = v & ~_mask_at(donor_masks[slot].cpu(), dx, dy)
                else:
                    bx = R[REC["paste_box"]:REC["paste_box"] + 4]
                    v = v & ~((dx >= bx[0]) & (dx <= bx[2]) & (dy >= bx[1]) & (dy <= bx[3]))
        else:
            v = _mask_at(donor_masks[-(s + 2)].cpu(), dx, dy)
        out[n] = v.to(torch.uint8)
    return out


def normalize_images(images: torch.Tensor, out_dtype=torch.bfloat16) -> torch.Tensor:
    """[B,3,H,W] uint8 or fp32 in [0,1] -> ImageNet-normalised ``out_dtype`` (CUDA kernel on the device)."""
    if images.is_cuda:
        out = torch.empty(images.shape, dtype=out_dtype, device=images.device)
        kernels().augment_images(images.contiguous(), out)
        return out
    return augment_reference(images).to(out_dtype)


# ------------------------------------------------------------------ the augmenter

class GpuAugmenter:
    """Per-rank augmenter: host planning + fused device pass.

    ``prepare(indices, reader, epoch, sequence)`` does the host work of one
    batch (plans, targets, mask decode) into pinned staging;
    ``apply(images, prepared)`` queues the uploads, the fused kernel, the mask
    warp and the donor-cache refresh on the current stream and returns
    ``(model_input, targets)`` on the device.  Without CUDA, ``apply`` runs the
    torch restatement.
    """

    def __init__(self, config: AugmentConfig, capacity: int, height: int, width: int, slots: int,
                 device: Optional[torch.device] = None, masks: bool = False, seed: int = 42, rank: int = 0,
                 out_dtype: torch.dtype = torch.bfloat16):
        self.config = config
        self.capacity, self.H, self.W, self.T = capacity, height, width, slots
        self.device = torch.device(device) if device is not None else torch.device("cpu")
        self.cuda = self.device.type == "cuda"
        self.masks = masks
        self.seed, self.rank = seed, rank
        self.out_dtype = out_dtype
        self.planner = native().AugmentPlanner(config_to_native(config), capacity, width, height, masks)
        pin = self.cuda
        self._ring = [self._staging(pin) for _ in range(2)]
        self._turn = 0
        dev = self.device
        self.records = torch.empty(capacity, REC["floats"], device=dev)
        self.out = torch.empty(capacity, 3, height, width, dtype=out_dtype, device=dev)
        self.donors = (torch.zeros(capacity, 3, height, width, dtype=torch.uint8, device=dev)
                       if _copy_paste_on(config) else None)
        self.donor_masks = (torch.zeros(capacity, height, width, dtype=torch.uint8, device=dev)
                            if (_copy_paste_on(config) and masks) else torch.zeros(0, height, width, dtype=torch.uint8,
                                                                                  device=dev))

    def _staging(self, pin: bool) -> dict:
        B, T = self.capacity, self.T
        s = dict(rec=torch.empty(B, REC["floats"], pin_memory=pin), boxes=torch.empty(B, T, 4, pin_memory=pin),
                 labels=torch.empty(B, T, dtype=torch.int64, pin_memory=pin),
                 counts=torch.empty(B, dtype=torch.int32, pin_memory=pin), areas=torch.empty(B, T, pin_memory=pin),
                 rows=torch.empty(B, T, dtype=torch.int32, pin_memory=pin), event=None, masks=None)
        return s

    def prepare(self, indices: Sequence[int], reader, epoch: int, sequence: int) -> dict:
        st = self._ring[self._turn]
        self._turn ^= 1
        if st["event"] is not None:
            st["event"].synchronize()   # this staging slot's previous uploads have finished
        n = len(indices)
        self.planner.plan(list(indices), self.seed, epoch, self.rank, sequence, st["rec"])
        pairs = self.planner.build_targets(reader, self.T, st["boxes"], st["labels"], st["counts"], st["areas"],
                                           st["rows"] if self.masks else None)
        if self.masks:
            need = max(1, len(pairs))
            if st["masks"] is None or st["masks"].shape[0] < need:
                st["masks"] = torch.empty(need, self.H, self.W, dtype=torch.uint8, pin_memory=self.cuda)
            reader.instance_masks(pairs, st["masks"])
        st["n"] = n
        st["pairs"] = len(pairs)
        st["replace"] = list(self.planner.replacements())
        if _TRACE_FILE:
            self._trace(indices, epoch, sequence, st)
        return st

    def _trace(self, indices, epoch: int, sequence: int, st: dict) -> None:
        """One JSONL record per batch (env ``MMLTK_AUGMENT_TRACE_FILE``; reference
        `src/rfdetr/gpu_augment.cpp:268-273`): the planned parameters of every image."""
        rec = st["rec"][:st["n"]]
        imgs = []
        for j, idx in enumerate(indices):
            r = rec[j]
            imgs.append({"index": int(idx), "augmented": bool(r[REC["flags"]] != 0),
                         "forward_affine": [round(float(v), 6) for v in r[REC["fwd"]:REC["fwd"] + 6]],
                         "color": [round(float(v), 6) for v in r[REC["color"]:REC["color"] + 9]],
                         "noise_mode": int(r[REC["noise_mode"]]), "noise_strength": round(float(r[REC["noise_str"]]), 6),
                         "blur": round(float(r[REC["blur"]]), 6), "occlusion_mode": int(r[REC["occ_mode"]]),
                         "paste_slot": int(r[REC["paste_slot"]]),
                         "targets": int(st["counts"][j])})
        line = {"rank": self.rank, "epoch": int(epoch), "sequence": int(sequence), "images": imgs}
        with open(_TRACE_FILE, "a") as f:
            f.write(json.dumps(line) + "\n")

    def apply(self, images: torch.Tensor, st: dict) -> Tuple[torch.Tensor, Targets]:
        n = st["n"]
        dev = self.device
        nb = self.cuda
        rec = self.records[:n]
        rec.copy_(st["rec"][:n], non_blocking=nb)
        counts_host = st["counts"][:n].tolist()
        tg = Targets(st["boxes"][:n].to(dev, non_blocking=nb), st["labels"][:n].to(dev, non_blocking=nb),
                     st["counts"][:n].to(dev, non_blocking=nb), counts_host)
        src = None
        if self.masks:
            src = st["masks"][:max(1, st["pairs"])].to(dev, non_blocking=nb)
            rows_host = st["rows"][:n]
            table = [(b, int(rows_host[b, t])) for b in range(n) for t in range(counts_host[b])]
            rows = torch.tensor(table if table else [[0, 0]], dtype=torch.int32)[:len(table)]
            if self.cuda:
                tg.masks = kernels().warp_masks(src, self.donor_masks, rows.to(dev), rec).bool()
            else:
                tg.masks = warp_masks_reference(src, self.donor_masks, rows, rec).bool()
            tg.mask_offsets = [0] + list(torch.tensor(counts_host).cumsum(0)[:-1].tolist()) if n else []
        if self.cuda:
            out = self.out[:n]
            kernels().augment_images(images.contiguous(), out, rec, self.donors,
                                     self.donor_masks if self.donor_masks.numel() else None)
        else:
            out = augment_reference(images, st["rec"][:n], self.donors,
                                    self.donor_masks if self.donor_masks.numel() else None).to(self.out_dtype)
        # donor cache refresh: queued after the kernel that read the old donors (same stream)
        for b, row in st["replace"]:
            if self.donors is not None:
                self.donors[b].copy_(images[b] if images.dtype == torch.uint8 else (images[b] * 255).round().byte())
            if self.masks and row >= 0 and self.donor_masks.numel():
                self.donor_masks[b].copy_(src[row])
        self.planner.commit_donors()
        if self.cuda:
            ev = torch.cuda.Event()
            ev.record()
            st["event"] = ev
        return out, tg
