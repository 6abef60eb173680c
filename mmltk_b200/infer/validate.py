"""Backend validation on a compiled split (reference `src/rfdetr/inference/validate.cpp:423-650`).

The reference compares its ONNX Runtime and TensorRT backends: COCO AP of each, timing, a
top-1 alignment probe (score, box and mask differences of every image's best detection) and the
AP delta.  Neither runtime is part of this environment, so the two backends compared here are

* ``native``: the B200 predictor (bf16, sm_100a kernels, CUDA graph) -- what `predict` runs;
* ``export``: the same weights through the export graph, the fp32 model on the CPU with the
  reference operator forms (grid-sample MSDeformAttn, softmax attention) -- the graph that
  ``export-onnx`` traces, so this is what an ONNX / TensorRT engine built from it computes.

The report keeps the reference's keys (``eval_order``, one summary per backend, ``alignment_probe``,
``delta_<second>_minus_<first>``).
"""
from __future__ import annotations

import copy
import time
from typing import Dict, List, Optional, Sequence

import torch

__all__ = ["validate_compiled"]


def _run(predictor, compiled: str, batch_size: int, max_dets: int, limit: Optional[int], workers: int):
    from ..data.loader import BatchLoader
    from ..eval import CocoEvaluator
    ev = CocoEvaluator(compiled, masks=predictor.with_masks, max_dets=max_dets)
    bl = BatchLoader(compiled, batch_size, shuffle=False, pixels="uint8", workers=workers, max_targets=1,
                     device=predictor.device if predictor.cuda else None)
    top1: Dict[int, dict] = {}
    n = 0
    t0 = time.perf_counter()
    for images, _t, idx in bl:
        if images.shape[0] != batch_size and predictor.use_graph:
            pad = torch.zeros(batch_size - images.shape[0], *images.shape[1:], dtype=images.dtype,
                              device=images.device)
            res = {k: v[:len(idx)] for k, v in predictor(torch.cat([images, pad])).items()}
        else:
            res = predictor(images)
        ev.add(idx, res["scores"], res["labels"], res["boxes"], res.get("masks"))
        for j, i in enumerate(idx):
            k = int(res["scores"][j].argmax())
            top1[int(i)] = {"score": float(res["scores"][j, k]), "label": int(res["labels"][j, k]),
                            "box": res["boxes"][j, k].float().cpu(),
                            "mask": None if "masks" not in res else res["masks"][j, k].bool().cpu()}
        n += len(idx)
        if limit and n >= limit:
            break
    if predictor.cuda:
        torch.cuda.synchronize(predictor.device)
    dt = time.perf_counter() - t0
    summary = ev.summarize()
    out = {"images": n, "seconds": dt, "img_per_s": n / dt if dt > 0 else 0.0,
           "bbox_ap": summary["bbox"]["ap"], "bbox_ap50": summary["bbox"]["ap50"],
           "bbox_ap75": summary["bbox"]["ap75"]}
    if "segm" in summary:
        out.update(mask_ap=summary["segm"]["ap"], mask_ap50=summary["segm"]["ap50"], mask_ap75=summary["segm"]["ap75"])
    else:
        out.update(mask_ap=None, mask_ap50=None, mask_ap75=None)
    return out, top1


def _alignment(a: Dict[int, dict], b: Dict[int, dict]) -> dict:
    common = sorted(set(a) & set(b))
    sd, bd, md = [], [], []
    for i in common:
        sd.append(abs(a[i]["score"] - b[i]["score"]))
        bd.append(float((a[i]["box"] - b[i]["box"]).abs().max()))
        if a[i]["mask"] is not None and b[i]["mask"] is not None:
            md.append(int((a[i]["mask"] ^ b[i]["mask"]).sum()))

    def stats(v):
        return (sum(v) / len(v), max(v)) if v else (None, None)
    s_mean, s_max = stats(sd)
    b_mean, b_max = stats(bd)
    m_mean, m_max = stats(md)
    return {"images_compared": len(common), "top1_score_abs_diff_mean": s_mean, "top1_score_abs_diff_max": s_max,
            "top1_box_abs_diff_px_mean": b_mean, "top1_box_abs_diff_px_max": b_max,
            "top1_mask_xor_pixels_mean": m_mean, "top1_mask_xor_pixels_max": m_max}


def validate_compiled(model, compiled: str, backends: Sequence[str] = ("native", "export"), batch_size: int = 1,
                      max_dets: int = 500, limit: Optional[int] = None, export_limit: Optional[int] = 16,
                      device=None, workers: int = 2) -> dict:
    """COCO AP, timing and top-1 alignment of ``backends`` on a compiled split.  ``export`` runs on
    the CPU in fp32 and is slow at full resolution, so it scores the first ``export_limit``
    images (the native backend is then scored on the same images)."""
    from .predictor import Predictor
    device = torch.device(device) if device is not None else (
        torch.device("cuda", 0) if torch.cuda.is_available() else torch.device("cpu"))
    n_limit = limit
    if "export" in backends and export_limit:
        n_limit = min(limit, export_limit) if limit else export_limit
    report: dict = {"batch_size": batch_size, "eval_order": list(backends)}
    tops: List[Dict[int, dict]] = []
    for name in backends:
        if name == "native":
            pred = Predictor(copy.deepcopy(model), device=device)
        elif name == "export":
            pred = Predictor(copy.deepcopy(model).float(), device="cpu", dtype=torch.float32, cuda_graph=False)
        else:
            raise ValueError(f"unknown validation backend {name!r} (native | export; ONNX Runtime and "
                             "TensorRT are not installed in this environment)")
        summary, top1 = _run(pred, compiled, batch_size, max_dets, n_limit, workers)
        if hasattr(pred, "release"):
            pred.release()
        report[name] = summary
        tops.append(top1)
        report["images"] = summary["images"]
    if len(backends) >= 2:
        report["alignment_probe"] = _alignment(tops[0], tops[1])
        a, b = report[backends[0]], report[backends[1]]
        report[f"delta_{backends[1]}_minus_{backends[0]}"] = {
            k: (None if a[k] is None or b[k] is None else b[k] - a[k])
            for k in ("bbox_ap", "bbox_ap50", "mask_ap", "mask_ap50")}
    return report
