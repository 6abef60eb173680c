"""Live frame analysis (headless).

Counterpart of the reference's live predict / frame analyzer
(`src/rfdetr/inference/live_predict.cpp:40-298`, lease rings and the
compositor of `src/live/*`): a capture thread writes frames into pinned slots
of a latest-frame lease ring (C++, ``csrc/host/lease_ring.cpp``); the analysis
loop leases the newest frame, uploads it, letterboxes + normalises it on the
GPU (one kernel), runs the CUDA-graph predictor, maps boxes back to the frame
and draws masks / boxes / labels on the device copy.  Display surfaces
(DMA-BUF/EGL interop, the browser compositor) are not available here: the
annotated frame stays a device buffer and can be written to PNG files.
"""
from __future__ import annotations

import dataclasses
import os
import threading
import time
from typing import Dict, Iterable, Optional, Sequence

import torch

from ..infer.predictor import Predictor
from ..infer.visualize import draw_detections, letterbox, letterbox_geometry
from ..ops._ext import native

__all__ = ["FrameAnalyzer", "LiveStats", "run_live"]


@dataclasses.dataclass
class LiveStats:
    frames_in: int = 0
    frames_analyzed: int = 0
    dropped: int = 0
    seconds: float = 0.0
    latency_ms_p50: float = 0.0

    @property
    def fps(self) -> float:
        return self.frames_analyzed / self.seconds if self.seconds > 0 else 0.0


class FrameAnalyzer:
    def __init__(self, predictor: Predictor, class_names: Sequence[str] = (), threshold: float = 0.5,
                 bgr: bool = True, draw: bool = True):
        self.p = predictor
        self.class_names = list(class_names)
        self.threshold = threshold
        self.bgr = bgr
        self.draw = draw
        self.H, self.W = predictor.size

    @torch.no_grad()
    def __call__(self, frame: torch.Tensor) -> Dict:
        """frame [h, w, 3] uint8 (host or device) -> dict(result, image)."""
        dev = self.p.device
        f = frame.to(dev, non_blocking=True)
        x = letterbox(f, self.H, self.W, self.bgr, normalize_bf16=self.p.cuda)[None]
        if not self.p.cuda:
            x = x.float()
        res = self.p(x)
        res = {k: v[0] for k, v in res.items()}
        s, tx, ty = letterbox_geometry(tuple(frame.shape[:2]), (self.H, self.W))
        b = res["boxes"].clone()
        b[:, 0::2] = ((b[:, 0::2] - tx) / s).clamp(0, frame.shape[1] - 1)
        b[:, 1::2] = ((b[:, 1::2] - ty) / s).clamp(0, frame.shape[0] - 1)
        res["boxes"] = b
        res.pop("masks", None)   # masks are predicted on the letterboxed canvas
        img = f
        if self.draw:
            img = f.clone()
            img = draw_detections(img, res, self.class_names, self.threshold, bgr=self.bgr)
        return {"result": res, "image": img}


def run_live(source: Iterable[torch.Tensor], analyzer: FrameAnalyzer, max_frames: Optional[int] = None,
             slots: int = 3, out_dir: Optional[str] = None, save_every: int = 0) -> LiveStats:
    """Capture thread -> lease ring -> analysis loop, until the source ends (or max_frames)."""
    it = iter(source)
    first = next(it)
    h, w, _ = first.shape
    pin = torch.cuda.is_available()
    bufs = [torch.empty(h, w, 3, dtype=torch.uint8, pin_memory=pin) for _ in range(slots)]
    ring = native().LeaseRing(slots)
    stats = LiveStats()
    done = threading.Event()

    def capture():
        seq = 0
        frame = first
        try:
            while frame is not None and not done.is_set():
                slot = ring.acquire_write()
                while slot < 0 and not done.is_set():
                    time.sleep(0.001)
                    slot = ring.acquire_write()
                if slot < 0:
                    break
                bufs[slot].copy_(frame)
                ring.publish(slot, seq)
                seq += 1
                stats.frames_in = seq
                if max_frames is not None and seq >= max_frames:
                    break
                frame = next(it, None)
        finally:
            ring.close()

    th = threading.Thread(target=capture, daemon=True)
    t0 = time.perf_counter()
    th.start()
    lat = []
    if out_dir:
        os.makedirs(out_dir, exist_ok=True)
    while True:
        got = ring.acquire_latest(2.0)
        if got is None:
            if not th.is_alive():
                break
            continue
        slot, seq = got
        ts = time.perf_counter()
        out = analyzer(bufs[slot])
        if analyzer.p.cuda:
            torch.cuda.current_stream().synchronize()
        ring.release(slot)
        lat.append((time.perf_counter() - ts) * 1e3)
        stats.frames_analyzed += 1
        if out_dir and save_every and stats.frames_analyzed % save_every == 0:
            img = out["image"].cpu()
            if analyzer.bgr:
                img = img.flip(-1)
            with open(os.path.join(out_dir, f"frame_{seq:06d}.png"), "wb") as fh:
                fh.write(native().encode_png(img.contiguous()))
    done.set()
    th.join(timeout=5)
    stats.seconds = time.perf_counter() - t0
    stats.dropped = int(ring.dropped())
    if lat:
        stats.latency_ms_p50 = float(torch.tensor(lat).median())
    return stats
