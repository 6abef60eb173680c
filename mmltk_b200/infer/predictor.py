"""Inference runtime: artifact resolution, a CUDA-graph predictor, compiled
dataset / image-file prediction with the reference's JSON output, evaluation.

Reference: `src/rfdetr/inference/predict.cpp:221-1081` (sources, staging, JSON
writer `:986-1025`, evaluation `:388-430,1027-1081`), artifact resolution
`src/rfdetr/layers/model.cpp:1529-1641`, record schema
`src/rfdetr/inference/predict_workflow_helpers.h:195-225`.

B200 design: one native backend.  The whole batch step -- uint8 pixels ->
normalised bf16 (fused kernel), the model in bf16, the fused top-k
post-process -- is captured once per batch shape in a CUDA graph and replayed;
a prediction costs one H2D copy of uint8 pixels, one replay and one D2H copy
of the top-k results.  Batch-1 latency is therefore launch-overhead free.
"""
from __future__ import annotations

import json
import os
import time
from typing import Dict, List, Optional, Sequence, Tuple

import torch

from ..ckpt import load_checkpoint, load_weights
from ..config.model_config import config_from_preset
from ..config.presets import find_preset, infer_preset_from_path
from ..data.augment import normalize_images
from ..models.rfdetr import RFDETR
from .postprocess import postprocess

__all__ = ["resolve_model", "Predictor", "predict_compiled", "predict_images", "write_predictions_json",
           "encode_mask_rle", "evaluate_compiled"]


def resolve_model(weights: Optional[str] = None, preset: Optional[str] = None, resolution: Optional[int] = None,
                  num_classes: Optional[int] = None, strict: bool = True, **overrides) -> Tuple[RFDETR, dict]:
    """Model config from (in order) the checkpoint's metadata, its file name,
    ``preset``; class count from the checkpoint unless given."""
    ckpt = load_checkpoint(weights) if weights else None
    name = None
    if ckpt is not None and ckpt.metadata.preset_name:
        name = ckpt.metadata.preset_name
    if name is None and weights:
        spec = infer_preset_from_path(weights)
        name = spec.name if spec else None
    name = name or preset
    if preset and name != preset and find_preset(preset) is not None:
        name = preset   # an explicit --preset wins over inference from the path
    if name is None or find_preset(name) is None:
        raise ValueError("cannot resolve the model preset: pass --preset")
    kw = dict(overrides)
    if resolution:
        kw["resolution"] = int(resolution)
    if num_classes is None and ckpt is not None and ckpt.metadata.num_classes:
        num_classes = ckpt.metadata.num_classes
    if num_classes is not None:
        kw["num_classes"] = int(num_classes)
    if ckpt is not None:
        for k, v in ckpt.metadata.optional.items():
            kw.setdefault(k, v)
    cfg = config_from_preset(name, **kw)
    model = RFDETR(cfg)
    info = {"preset_name": name, "weights_path": os.path.abspath(weights) if weights else "",
            "input_kind": "weights" if weights else "preset"}
    if ckpt is not None:
        summary = load_weights(model, ckpt, strict=strict)
        info["load_summary"] = {"loaded": len(summary.loaded), "missing": summary.missing,
                                "unexpected": summary.unexpected, "incompatible": summary.incompatible}
    return model, info


class Predictor:
    """Batched predictor.  ``images``: [B,3,H,W] uint8 (k/255) or fp32 in [0,1]."""

    def __init__(self, model: RFDETR, device="cuda", dtype: torch.dtype = torch.bfloat16,
                 num_select: Optional[int] = None, cuda_graph: bool = True, with_masks: Optional[bool] = None):
        self.device = torch.device(device)
        self.cuda = self.device.type == "cuda"
        self.dtype = dtype if self.cuda else torch.float32
        self.model = model.eval().to(device=self.device, dtype=self.dtype)
        if self.cuda and os.environ.get("MMLTK_CL_CONV_WEIGHTS", "1") != "0":
            # the convolutions run on channels-last activations; weights in the same layout spare
            # cuDNN a per-call weight transform (one copy kernel per 3x3 conv and forward)
            for mod in self.model.modules():
                if isinstance(mod, (torch.nn.Conv2d, torch.nn.ConvTranspose2d)) and mod.weight.dim() == 4 \
                        and mod.weight.shape[-1] * mod.weight.shape[-2] > 1:
                    mod.weight.data = mod.weight.data.contiguous(memory_format=torch.channels_last)
        self.cfg = model.cfg
        self.size = (self.cfg.resolution, self.cfg.resolution)
        self.k = int(num_select or self.cfg.num_select)
        self.with_masks = self.cfg.segmentation if with_masks is None else with_masks
        self.use_graph = cuda_graph and self.cuda
        self._graphs: Dict[Tuple, dict] = {}

    @torch.no_grad()
    def _step(self, images: torch.Tensor) -> Dict[str, torch.Tensor]:
        x = normalize_images(images, self.dtype) if images.dtype == torch.uint8 or images.dtype == torch.float32 \
            else images
        out = self.model(x, include_masks=self.with_masks)
        return postprocess(out, self.k, self.size, masks=self.with_masks)

    def _graph(self, images: torch.Tensor) -> dict:
        key = (tuple(images.shape), images.dtype)
        g = self._graphs.get(key)
        if g is None:
            static = torch.empty_like(images, device=self.device)
            static.copy_(images)
            s = torch.cuda.Stream(self.device)
            s.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(s):
                for _ in range(2):                  # warm-up: allocations, caches, autotuning outside capture
                    self._step(static)
            torch.cuda.current_stream(self.device).wait_stream(s)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                outs = self._step(static)
                # the host-bound results packed into one byte buffer inside the graph, so that
                # fetching them is one device-to-host copy (largest element size first: every
                # segment then starts aligned for its dtype)
                keys = sorted((k for k in outs if k != "masks"), key=lambda k: -outs[k].element_size())
                packed = torch.cat([outs[k].contiguous().view(torch.uint8).reshape(-1) for k in keys])
            layout, off = [], 0
            for k in keys:
                nb = outs[k].numel() * outs[k].element_size()
                layout.append((k, off, nb, outs[k].dtype, tuple(outs[k].shape)))
                off += nb
            host = torch.empty(packed.numel(), dtype=torch.uint8, pin_memory=True)
            g = {"graph": graph, "input": static, "outputs": outs, "packed": packed, "host": host, "layout": layout}
            self._graphs[key] = g
        return g

    @torch.no_grad()
    def __call__(self, images: torch.Tensor) -> Dict[str, torch.Tensor]:
        """Device results (graph path: the static buffers -- consume them before the next call)."""
        if not self.use_graph:
            return self._step(images.to(self.device, non_blocking=True))
        g = self._graph(images)
        g["input"].copy_(images, non_blocking=True)
        g["graph"].replay()
        return g["outputs"]

    @torch.no_grad()
    def predict_host(self, images: torch.Tensor) -> Dict[str, torch.Tensor]:
        """Results in host memory (masks excluded).  Graph path: one asynchronous copy of the
        packed results into a pinned buffer; the returned tensors are views of that buffer,
        valid until the next call."""
        if not self.use_graph:
            r = self(images)
            return {k: v.cpu() for k, v in r.items() if k != "masks"}
        self(images)
        g = self._graphs[(tuple(images.shape), images.dtype)]
        host = g["host"]
        host.copy_(g["packed"], non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        return {k: host[o:o + nb].view(dt).view(shape) for k, o, nb, dt, shape in g["layout"]}

    def release(self) -> None:
        self._graphs.clear()

    @torch.no_grad()
    def latency(self, iters: int = 100, warmup: int = 10, batch: int = 1, pin_cpus: bool = True) -> Dict[str, float]:
        """Batch-``batch`` latency percentiles (ms): pinned host uint8 input -> results in pinned
        host memory, bracketed by CUDA events.  ``pin_cpus``: run the calling thread on the GPU's
        own NUMA node while measuring (the host enqueues the copies and the graph replay, so its
        placement is on the critical path)."""
        x = torch.randint(0, 256, (batch, 3, *self.size), dtype=torch.uint8).pin_memory() if self.cuda else \
            torch.randint(0, 256, (batch, 3, *self.size), dtype=torch.uint8)
        saved = None
        if self.cuda and pin_cpus:
            from ..utils.runtime import gpu_local_cpus
            local = gpu_local_cpus(self.device)
            if local:
                saved = os.sched_getaffinity(0)
                os.sched_setaffinity(0, local)
        try:
            for _ in range(warmup):
                self.predict_host(x) if self.cuda else self(x)
            times = []
            for _ in range(iters):
                if self.cuda:
                    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    torch.cuda.synchronize(self.device)
                    a.record()
                    r = self(x)
                    if self.use_graph:
                        g = self._graphs[(tuple(x.shape), x.dtype)]
                        g["host"].copy_(g["packed"], non_blocking=True)
                    else:
                        r = {k: v.to("cpu", non_blocking=True) for k, v in r.items() if k != "masks"}
                    b.record()
                    b.synchronize()
                    times.append(a.elapsed_time(b))
                else:
                    t0 = time.perf_counter()
                    self(x)
                    times.append((time.perf_counter() - t0) * 1e3)
        finally:
            if saved is not None:
                os.sched_setaffinity(0, saved)
        t = torch.tensor(times)
        return {"p50_ms": float(t.median()), "p90_ms": float(t.quantile(0.9)), "p99_ms": float(t.quantile(0.99)),
                "mean_ms": float(t.mean()), "images_per_s": float(batch * 1e3 / t.mean()), "iters": iters,
                "batch": batch}


def encode_mask_rle(mask: torch.Tensor) -> str:
    """Row-major ``start:length`` runs of a binary [H,W] mask."""
    flat = mask.flatten().to(torch.int8)
    d = torch.diff(torch.cat([flat.new_zeros(1), flat, flat.new_zeros(1)]))
    starts = (d == 1).nonzero().flatten().tolist()
    ends = (d == -1).nonzero().flatten().tolist()
    return " ".join(f"{s}:{e - s}" for s, e in zip(starts, ends))


def _records(results: Dict[str, torch.Tensor], indices: Sequence[int], names: Sequence[str],
             class_names: Sequence[str], threshold: float) -> List[dict]:
    host = {k: v.cpu() for k, v in results.items()}
    recs = []
    for b, di in enumerate(indices):
        dets = []
        for j in range(host["scores"].shape[1]):
            s = float(host["scores"][b, j])
            if s < threshold:
                continue
            lab = int(host["labels"][b, j])
            d = {"label": class_names[lab] if 0 <= lab < len(class_names) and class_names[lab] else str(lab + 1),
                 "score": s, "xyxy": [float(v) for v in host["boxes"][b, j]]}
            if "masks" in host:
                d["mask_rle"] = encode_mask_rle(host["masks"][b, j])
            dets.append(d)
        r = {"dataset_index": int(di), "image_id": int(di) + 1, "detections": dets}
        if names and names[b]:
            r["source_name"] = names[b]
        recs.append(r)
    return recs


def _draw_batch(images, res, idx, class_names, threshold, out_dir) -> None:
    """Annotated PNGs (masks, boxes, label bars drawn on the device) for one batch."""
    from ..ops._ext import native
    from .visualize import draw_detections
    os.makedirs(out_dir, exist_ok=True)
    for j, di in enumerate(idx):
        img = images[j]
        if img.dtype != torch.uint8:
            img = (img.float() * 255).round().clamp(0, 255).to(torch.uint8)
        hwc = img.permute(1, 2, 0).contiguous()
        one = {k: v[j] for k, v in res.items()}
        hwc = draw_detections(hwc, one, class_names, threshold)
        with open(os.path.join(out_dir, f"{int(di):06d}.png"), "wb") as f:
            f.write(native().encode_png(hwc.cpu()))


def predict_compiled(predictor: Predictor, compiled: str, batch_size: int = 1, threshold: float = 0.5,
                     workers: int = 4, limit: Optional[int] = None, evaluator=None,
                     draw_dir: Optional[str] = None) -> Tuple[List[dict], dict]:
    from ..data.loader import BatchLoader
    bl = BatchLoader(compiled, batch_size, shuffle=False, pixels="uint8", workers=workers, max_targets=1,
                     device=predictor.device if predictor.cuda else None)
    class_names = bl.dataset.class_names
    records: List[dict] = []
    n = 0
    t0 = time.perf_counter()
    for images, _targets, idx in bl:
        if images.shape[0] != batch_size and predictor.use_graph:
            pad = torch.zeros(batch_size - images.shape[0], *images.shape[1:], dtype=images.dtype,
                              device=images.device)
            res = predictor(torch.cat([images, pad]))
            res = {k: v[:len(idx)] for k, v in res.items()}
        else:
            res = predictor(images)
        if evaluator is not None:
            evaluator.add(idx, res["scores"], res["labels"], res["boxes"], res.get("masks"))
        if draw_dir:
            _draw_batch(images, res, idx, class_names, threshold, draw_dir)
        records += _records(res, idx, [], class_names, threshold)
        n += len(idx)
        if limit and n >= limit:
            break
    if predictor.cuda:
        torch.cuda.synchronize(predictor.device)
    dt = time.perf_counter() - t0
    return records, {"images": n, "seconds": dt, "img_per_s": n / dt if dt > 0 else 0.0}


def predict_images(predictor: Predictor, paths: Sequence[str], threshold: float = 0.5) -> List[dict]:
    from ..ops._ext import native
    H, W = predictor.size
    records = []
    for i, p in enumerate(paths):
        with open(p, "rb") as f:
            rgb = native().decode_png(f.read())                       # [h, w, 3] uint8
        x = rgb.permute(2, 0, 1)[None].float()
        if tuple(x.shape[-2:]) != (H, W):
            x = torch.nn.functional.interpolate(x, size=(H, W), mode="area" if x.shape[-1] >= W else "bilinear")
        x = (x / 255.0).clamp(0, 1)
        res = predictor(x.to(predictor.device))
        # boxes back to the source image's pixels
        sx, sy = rgb.shape[1] / W, rgb.shape[0] / H
        res = dict(res)
        res["boxes"] = res["boxes"] * torch.tensor([sx, sy, sx, sy], device=res["boxes"].device)
        res.pop("masks", None) if (rgb.shape[0], rgb.shape[1]) != (H, W) else None
        records += _records(res, [i], [os.path.basename(p)], [], threshold)
    return records


def write_predictions_json(path: str, records: List[dict], info: dict, source_kind: str,
                           compiled_path: Optional[str] = None, image_count: Optional[int] = None,
                           backend: str = "native-b200") -> None:
    payload = {"source_kind": source_kind, "model_kind": info.get("input_kind", "weights"),
               "model_path": info.get("weights_path", ""), "preset_name": info.get("preset_name", ""),
               "backend": backend, "mask_rle_encoding": "row_major_start_length", "records": records}
    if compiled_path is not None:
        payload["compiled_path"] = compiled_path
    if image_count is not None:
        payload["input_image_count"] = image_count
    if info.get("weights_path"):
        payload["weights_path"] = info["weights_path"]
    os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
    with open(path, "w") as f:
        json.dump(payload, f, indent=2)
        f.write("\n")


def evaluate_compiled(predictor: Predictor, compiled: str, batch_size: int = 8, max_dets: int = 500,
                      workers: int = 4) -> dict:
    from ..eval import CocoEvaluator
    ev = CocoEvaluator(compiled, masks=predictor.with_masks, max_dets=max_dets)
    _, timing = predict_compiled(predictor, compiled, batch_size, threshold=1.1, workers=workers, evaluator=ev)
    out = ev.summarize()
    out["images"] = ev.num_images
    out["timing"] = timing
    return out
