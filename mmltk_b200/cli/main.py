"""``mmltk`` command line.

Commands (reference `src/cli.cpp:144-245`, `src/rfdetr/cli/cli.cpp:185-454`,
options `src/rfdetr/cli/workflow_cli_shared.h:75-648`, request validation
`src/rfdetr/workflow_requests.cpp:58-345`):

* ``mmltk compile|info|bench`` -- compiled datasets;
* ``mmltk rfdetr compile|info|train|predict|evaluate|export-onnx|build-engine|
  normalize-weights|validate|latency``.

``train --device-ids 0,1,...`` forks one worker per device (``--dist-*``
flags are the internal worker protocol).  ``--compile-mode none`` runs the
training step eagerly; ``selective`` / ``full`` capture it in a CUDA graph
(this framework's replacement for TorchScript tracing).  TensorRT and ONNX
Runtime are not part of this environment: ``build-engine`` and the ONNX/TRT
backends of ``predict`` / ``evaluate`` / ``validate`` report that and exit 2.
"""
from __future__ import annotations

import argparse
import json
import logging
import os
import sys
from typing import List, Optional

__all__ = ["main", "build_parser", "train_options_from_args"]

log = logging.getLogger("mmltk")


class Unavailable(RuntimeError):
    pass


def _bool_flag(p, name, dest, default, help_):
    p.add_argument(f"--{name}", dest=dest, action="store_true", default=default, help=help_)
    p.add_argument(f"--no-{name}", dest=dest, action="store_false")


def _add_compile(p):
    p.add_argument("--source", required=True, help="source dataset directory (categories.json + split dirs)")
    p.add_argument("--output", required=True, help="output directory for <split>.bin")
    p.add_argument("--splits", default=None, help="comma-separated split names (default: every subdirectory)")
    p.add_argument("--resolution", type=int, default=0, help="square output size (overrides width/height)")
    p.add_argument("--width", type=int, default=432)
    p.add_argument("--height", type=int, default=432)
    p.add_argument("--workers", type=int, default=0)
    p.add_argument("--cuda-mask-batch-size", type=int, default=0, help="accepted for compatibility (masks are "
                   "resized on the host thread pool)")


def _add_model_inputs(p):
    p.add_argument("--weights", default=None)
    p.add_argument("--onnx", default=None)
    p.add_argument("--tensorrt", default=None)
    p.add_argument("--preset", default=None)
    p.add_argument("--resolution", type=int, default=0)


def _add_execution(p):
    p.add_argument("--device-id", type=int, default=0)
    p.add_argument("--workers", type=int, default=4)
    p.add_argument("--lanes", type=int, default=1)
    p.add_argument("--cpu-affinity", default="")
    p.add_argument("--batch-size", type=int, default=1)
    p.add_argument("--compile-mode", choices=("none", "selective", "full"), default="selective")
    _bool_flag(p, "fp16", "fp16", True, "reduced-precision inference (bf16 on B200)")
    _bool_flag(p, "progress", "progress", False, "progress output")


def _add_aug_group(p, name):
    p.add_argument(f"--aug-{name}-prob", type=float, default=None)
    p.add_argument(f"--aug-{name}-min-strength", type=float, default=None)
    p.add_argument(f"--aug-{name}-max-strength", type=float, default=None)


def _add_train(p):
    g = p.add_argument_group("Dataset")
    g.add_argument("--train-compiled")
    g.add_argument("--val-compiled")
    g.add_argument("--test-compiled")
    g.add_argument("--resolution", type=int, default=0)
    g = p.add_argument_group("Checkpoint")
    g.add_argument("--output-dir")
    g.add_argument("--weights")
    g.add_argument("--resume")
    g.add_argument("--preset", default="")
    g = p.add_argument_group("Optimization")
    g.add_argument("--batch-size", type=int, default=None)
    g.add_argument("--val-batch-size", type=int, default=None)
    g.add_argument("--epochs", type=int, default=None)
    g.add_argument("--grad-accum-steps", type=int, default=None)
    g.add_argument("--optimizer", choices=("adamw", "muon"), default="adamw")
    for f in ("lr", "lr-encoder", "momentum", "lr-component-decay", "encoder-layer-decay", "weight-decay",
              "lr-min-factor", "warmup-epochs", "warmup-momentum", "clip-max-norm", "ema-decay"):
        g.add_argument(f"--{f}", type=float, default=None)
    g.add_argument("--lr-drop", type=int, default=None)
    g.add_argument("--lr-scheduler", choices=("step", "cosine"), default=None)
    g.add_argument("--ema-tau", type=int, default=None)
    g.add_argument("--eval-max-dets", type=int, default=None)
    _bool_flag(g, "freeze-encoder", "freeze_encoder", None, "freeze the encoder")
    _bool_flag(g, "fused-optimizer", "fused_optimizer", None, "fused AdamW kernels")
    _bool_flag(g, "use-ema", "use_ema", None, "EMA shadow model")
    g.add_argument("--no-ema", dest="use_ema", action="store_false")
    _bool_flag(g, "validation-loss", "validation_loss", None, "criterion loss on the validation split")
    _bool_flag(g, "validation-profile", "validation_profile", None, "validation JSONL phase records")
    g = p.add_argument_group("GPU augmentation")
    _bool_flag(g, "gpu-augment", "gpu_augment", None, "fused GPU training augmentation")
    for name in ("geometry", "resize", "color", "noise", "blur", "occlusion"):
        _add_aug_group(g, name)
    g.add_argument("--aug-copy-paste-prob", type=float, default=None)
    g = p.add_argument_group("Execution")
    g.add_argument("--device-id", type=int, default=0)
    g.add_argument("--device-ids", default="")
    g.add_argument("--workers", type=int, default=0)
    g.add_argument("--lanes", type=int, default=0)
    g.add_argument("--cpu-affinity", default="", help="CPU list for this run, e.g. 0-15,32-47 (ranks get shards)")
    _bool_flag(g, "high-priority", "high_priority", None,
               "lowest permitted nice value and realtime I/O priority (best effort)")
    g.add_argument("--prefetch-factor", type=int, default=None)
    g.add_argument("--print-freq", type=int, default=None)
    g.add_argument("--seed", type=int, default=None)
    _bool_flag(g, "amp", "amp", None, "mixed precision (bf16)")
    g.add_argument("--compile-mode", choices=("none", "selective", "full"), default=None)
    g.add_argument("--ddp-backend", choices=("fused", "nccl"), default=None,
                   help="multi-GPU gradient step: in-kernel NVSwitch (fused) or NCCL all-reduce")
    g = p.add_argument_group("Distributed (internal)")
    g.add_argument("--dist-worker", action="store_true")
    g.add_argument("--dist-rank", type=int, default=0)
    g.add_argument("--dist-world-size", type=int, default=1)
    g.add_argument("--dist-store-file", default="")


def build_parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(prog="mmltk", description="B200-native RF-DETR training and inference")
    ap.add_argument("--log-level", default=os.environ.get("MMLTK_LOG_LEVEL", "info"))
    ap.add_argument("--log-file", default=os.environ.get("MMLTK_LOG_FILE", ""))
    sub = ap.add_subparsers(dest="cmd", required=True)
    _add_compile(sub.add_parser("compile", help="compile a source dataset"))
    p = sub.add_parser("info", help="describe a compiled dataset")
    p.add_argument("path")
    sub.add_parser("models", help="registered model families, capabilities and presets")
    p = sub.add_parser("bench", help="loader throughput of a compiled dataset")
    p.add_argument("path")
    p.add_argument("--batch-size", type=int, default=8)
    p.add_argument("--batches", type=int, default=50)
    p.add_argument("--workers", type=int, default=4)

    rf = sub.add_parser("rfdetr", help="RF-DETR workflows").add_subparsers(dest="rcmd", required=True)
    _add_compile(rf.add_parser("compile"))
    p = rf.add_parser("info", help="describe a compiled dataset, checkpoint or ONNX model")
    p.add_argument("path")
    _add_train(rf.add_parser("train"))
    p = rf.add_parser("predict")
    p.add_argument("images", nargs="*")
    p.add_argument("--compiled")
    p.add_argument("--output", required=True)
    p.add_argument("--threshold", type=float, default=0.5)
    p.add_argument("--backend", choices=("auto", "weights", "onnx", "tensorrt"), default="auto")
    p.add_argument("--draw-dir", default=None, help="write annotated PNGs (drawn on the GPU) here")
    _add_model_inputs(p)
    _add_execution(p)
    p = rf.add_parser("evaluate")
    p.add_argument("--compiled", required=True)
    p.add_argument("--output", default=None)
    p.add_argument("--max-dets", type=int, default=500)
    p.add_argument("--backend", choices=("auto", "weights", "onnx", "tensorrt"), default="auto")
    _add_model_inputs(p)
    _add_execution(p)
    p = rf.add_parser("export-onnx")
    p.add_argument("--output", required=True)
    p.add_argument("--opset-version", type=int, default=19)
    p.add_argument("--simplify", action="store_true")
    p.add_argument("--batch-size", type=int, default=1)
    p.add_argument("--device-id", type=int, default=0)
    _add_model_inputs(p)
    p = rf.add_parser("build-engine")
    p.add_argument("--onnx", required=True)
    p.add_argument("--output", required=True)
    _bool_flag(p, "fp16", "fp16", True, "FP16 engine")
    p = rf.add_parser("normalize-weights")
    p.add_argument("--input", "--weights", dest="input", required=True)
    p.add_argument("--output", required=True)
    p = rf.add_parser("validate", help="native B200 predictor vs the export graph (fp32, CPU) on a compiled split")
    p.add_argument("--compiled")
    p.add_argument("--source")
    p.add_argument("--output", default=None)
    p.add_argument("--max-dets", type=int, default=500)
    p.add_argument("--limit", type=int, default=None, help="score only the first N images")
    p.add_argument("--export-limit", type=int, default=16,
                   help="images scored by the export backend (fp32 on the CPU); both backends use them")
    _add_model_inputs(p)
    _add_execution(p)
    p = rf.add_parser("live", help="headless live analysis of a frame source (synthetic: no capture device)")
    _add_model_inputs(p)
    p.add_argument("--synthetic", action="store_true", default=True)
    p.add_argument("--frames", type=int, default=300)
    p.add_argument("--width", type=int, default=1280)
    p.add_argument("--height", type=int, default=720)
    p.add_argument("--threshold", type=float, default=0.5)
    p.add_argument("--output", default=None, help="directory for annotated PNG frames")
    p.add_argument("--save-every", type=int, default=0)
    p.add_argument("--device-id", type=int, default=0)
    p = rf.add_parser("latency", help="batch-1 (or --batch-size) latency of the CUDA-graph predictor")
    _add_model_inputs(p)
    p.add_argument("--batch-size", type=int, default=1)
    p.add_argument("--iters", type=int, default=200)
    p.add_argument("--device-id", type=int, default=0)
    p.add_argument("--device-ids", default="", help="e.g. 0,1,...,7: one replica per GPU, concurrent throughput")
    p.add_argument("--no-pin-cpus", action="store_true",
                   help="do not run the measuring thread on the GPU's NUMA-local CPUs")
    return ap


# ------------------------------------------------------------------ train options

_SIMPLE = {"batch_size": "batch_size", "val_batch_size": "val_batch_size", "epochs": "epochs",
           "grad_accum_steps": "grad_accum_steps", "lr": "lr", "lr_encoder": "lr_encoder", "momentum": "momentum",
           "lr_component_decay": "lr_component_decay", "encoder_layer_decay": "encoder_layer_decay",
           "weight_decay": "weight_decay", "lr_min_factor": "lr_min_factor", "warmup_epochs": "warmup_epochs",
           "warmup_momentum": "warmup_momentum", "clip_max_norm": "clip_max_norm", "ema_decay": "ema_decay",
           "lr_drop": "lr_drop", "lr_scheduler": "lr_scheduler", "ema_tau": "ema_tau",
           "eval_max_dets": "eval_max_dets", "freeze_encoder": "freeze_encoder",
           "fused_optimizer": "fused_optimizer", "use_ema": "use_ema", "validation_loss": "validation_loss",
           "validation_profile": "validation_profile", "prefetch_factor": "prefetch_factor",
           "print_freq": "print_freq", "seed": "seed", "amp": "amp", "compile_mode": "compile_mode",
           "ddp_backend": "ddp_backend", "high_priority": "high_priority"}


def train_options_from_args(a) -> "TrainOptions":
    from ..config import TrainOptions, apply_recipe
    o = TrainOptions(train_compiled=a.train_compiled, val_compiled=a.val_compiled, test_compiled=a.test_compiled,
                     output_dir=a.output_dir, weights=a.weights, resume=a.resume, preset=a.preset or "",
                     resolution=a.resolution, optimizer=a.optimizer, device_id=a.device_id, workers=a.workers,
                     lanes=a.lanes, cpu_affinity=a.cpu_affinity, dist_worker=a.dist_worker, dist_rank=a.dist_rank,
                     dist_world_size=a.dist_world_size, dist_store_file=a.dist_store_file)
    o.device_ids = [int(x) for x in a.device_ids.split(",") if x.strip()] if a.device_ids else []
    for src, dst in _SIMPLE.items():
        v = getattr(a, src, None)
        if v is not None:
            setattr(o, dst, v)
            o.overrides.add(dst)
    apply_recipe(o)
    o.cuda_graph = o.compile_mode != "none"
    aug = o.augmentation
    if a.gpu_augment is not None:
        aug.enabled = a.gpu_augment
    for name in ("geometry", "resize", "color", "noise", "blur", "occlusion"):
        grp = getattr(aug, name)
        for suffix, field in (("prob", "probability"), ("min_strength", "min_strength"),
                              ("max_strength", "max_strength")):
            v = getattr(a, f"aug_{name}_{suffix}")
            if v is not None:
                setattr(grp, field, v)
    if a.aug_copy_paste_prob is not None:
        aug.copy_paste_probability = a.aug_copy_paste_prob
    o.validate()
    if not o.dist_worker:
        if not o.train_compiled or not o.val_compiled or not o.output_dir:
            raise SystemExit("train requires --train-compiled, --val-compiled and --output-dir")
        if o.weights and o.resume:
            raise SystemExit("train takes exactly one of --weights / --resume")
        if not (o.weights or o.resume or o.preset):
            raise SystemExit("train requires --weights, --resume or --preset")
    if o.optimizer == "muon":
        log.warning("optimizer=muon: the fused AdamW step is not used; Muon runs in its eager form")
    if o.lanes and o.lanes > 1:
        log.info("--lanes %d: each optimizer step sums the gradients of %d lane batches (x --grad-accum-steps), "
                 "run back to back on one stream as graph replays instead of model replicas", o.lanes, o.lanes)
    return o


# ------------------------------------------------------------------ commands

def _compile(a) -> int:
    from ..data.compiler import compile_dataset
    w, h = (a.resolution, a.resolution) if a.resolution else (a.width, a.height)
    splits = a.splits.split(",") if a.splits else None
    for st in compile_dataset(a.source, a.output, splits, w, h, a.workers):
        print(json.dumps(st))
    return 0


def _info(path: str) -> int:
    from ..ckpt import is_native_checkpoint
    if path.endswith(".onnx"):
        from ..export import onnx_info
        print(json.dumps(onnx_info(path), indent=1))
        return 0
    if path.endswith(".bin"):
        from ..data.loader import CompiledDataset
        ds = CompiledDataset(path)
        h = dict(ds.header)
        print(json.dumps(h, indent=1))
        return 0
    if is_native_checkpoint(path) or path.endswith((".pt", ".pth")):
        from ..ckpt import load_checkpoint
        ck = load_checkpoint(path)
        print(json.dumps({"preset_name": ck.metadata.preset_name, "source_kind": ck.metadata.source_kind,
                          "num_classes": ck.metadata.num_classes, "tensors": len(ck.state_dict),
                          "parameters": int(sum(t.numel() for t in ck.state_dict.values())),
                          "optional": ck.metadata.optional, "resume_keys": sorted(ck.extra)}, indent=1))
        return 0
    raise SystemExit(f"info: unknown file type: {path}")


def _bench(a) -> int:
    import time
    from ..data.loader import BatchLoader
    bl = BatchLoader(a.path, a.batch_size, shuffle=True, workers=a.workers, pixels="uint8", max_targets=1)
    t0, n = time.perf_counter(), 0
    for i, (images, _t, idx) in enumerate(bl):
        n += len(idx)
        if i + 1 >= a.batches:
            break
    dt = time.perf_counter() - t0
    print(json.dumps({"images": n, "seconds": dt, "images_per_second": n / dt if dt else 0.0}))
    return 0


def _require_native_backend(a) -> None:
    from ..models.registry import ModelArtifactRequest, default_registry
    req = ModelArtifactRequest(weights_path=a.weights or "", onnx_path=getattr(a, "onnx", None) or "",
                               tensorrt_path=getattr(a, "tensorrt", None) or "", preset_name=a.preset or "",
                               resolution=a.resolution or 0)
    try:
        req.validate()
    except ValueError as e:
        raise SystemExit(str(e))
    kind = req.selected_input_kind()
    if getattr(a, "backend", "auto") in ("onnx", "tensorrt"):
        kind = a.backend
    module = default_registry().find_module("rfdetr")
    caps = module.capabilities()
    if (kind == "onnx" and not caps.supports_onnx) or (kind == "tensorrt" and not caps.supports_tensorrt):
        raise Unavailable("ONNX Runtime and TensorRT are not installed in this environment; "
                          "use --weights (the native B200 backend)")


def _models() -> int:
    """Registered model families, their capabilities and presets (JSON)."""
    from dataclasses import asdict
    from ..models.registry import default_registry
    reg = default_registry()
    print(json.dumps([{"module_id": m.module_id, "display_name": m.display_name,
                       "capabilities": asdict(m.capabilities()),
                       "presets": [asdict(p) for p in m.presets()]} for m in reg.modules()], indent=1))
    return 0


def _predictor(a):
    import torch
    from ..infer import Predictor, resolve_model
    model, info = resolve_model(a.weights, preset=a.preset, resolution=a.resolution or None)
    dev = torch.device("cuda", a.device_id) if torch.cuda.is_available() else torch.device("cpu")
    cg = getattr(a, "compile_mode", "selective") != "none"
    return Predictor(model, device=dev, cuda_graph=cg), info


def _predict(a) -> int:
    from ..infer import predict_compiled, predict_images, write_predictions_json
    _require_native_backend(a)
    if bool(a.compiled) == bool(a.images):
        raise SystemExit("predict takes --compiled or image paths (exactly one source)")
    pred, info = _predictor(a)
    if a.compiled:
        recs, timing = predict_compiled(pred, a.compiled, a.batch_size, a.threshold, a.workers,
                                        draw_dir=a.draw_dir)
        write_predictions_json(a.output, recs, info, "compiled_dataset", compiled_path=a.compiled)
    else:
        recs = predict_images(pred, a.images, a.threshold)
        timing = {"images": len(recs)}
        write_predictions_json(a.output, recs, info, "image_files", image_count=len(a.images))
    print(f"rfdetr predict[native-b200]: preset={info['preset_name']} records={len(recs)} "
          f"threshold={a.threshold} output={a.output} timing={json.dumps(timing)}")
    return 0


def _evaluate(a) -> int:
    from ..infer import evaluate_compiled
    _require_native_backend(a)
    pred, info = _predictor(a)
    res = evaluate_compiled(pred, a.compiled, max(1, a.batch_size), a.max_dets, a.workers)
    b = res["bbox"]
    m = res.get("segm")
    print(f"rfdetr evaluate[native-b200]: preset={info['preset_name']} images={res['images']} "
          f"bbox_ap={b['ap']:.6f} bbox_ap50={b['ap50']:.6f} bbox_ap75={b['ap75']:.6f} "
          + (f"mask_ap={m['ap']:.6f} mask_ap50={m['ap50']:.6f} mask_ap75={m['ap75']:.6f}" if m else
             "mask_ap=null mask_ap50=null mask_ap75=null"))
    if a.output:
        with open(a.output, "w") as f:
            json.dump(res, f, indent=1)
    return 0


def _validate(a) -> int:
    from ..infer import resolve_model
    from ..infer.validate import validate_compiled
    if a.onnx or a.tensorrt or not a.weights and not a.preset:
        raise Unavailable("validate compares ONNX Runtime and TensorRT in the reference; neither is installed "
                          "in this environment -- pass --weights (or --preset) to compare the native B200 "
                          "predictor with the export graph instead")
    if not a.compiled:
        raise SystemExit("validate requires --compiled (a compiled split; --source recompilation is not supported)")
    model, info = resolve_model(a.weights, preset=a.preset, resolution=a.resolution or None)
    rep = validate_compiled(model, a.compiled, ("native", "export"), max(1, a.batch_size), a.max_dets, a.limit,
                            a.export_limit, workers=max(1, a.workers))
    rep["model"] = info.get("preset_name")
    print(json.dumps(rep, indent=1))
    if a.output:
        with open(a.output, "w") as f:
            json.dump(rep, f, indent=1)
    return 0


def _export(a) -> int:
    from ..export import export_onnx
    from ..infer import resolve_model
    if a.simplify:
        log.warning("--simplify: onnx-simplifier is not installed; exporting without simplification")
    model, _ = resolve_model(a.weights, preset=a.preset, resolution=a.resolution or None)
    print(json.dumps(export_onnx(model, a.output, a.opset_version, a.batch_size), indent=1))
    return 0


def _train(a) -> int:
    from ..parallel.launch import launch_workers
    from ..train.loop import run_training
    o = train_options_from_args(a)
    if len(o.device_ids) > 1 and not o.dist_worker:
        return launch_workers(a.raw_argv, o.device_ids, workers=o.workers, cpu_affinity=o.cpu_affinity)
    if len(o.device_ids) == 1:
        o.device_id = o.device_ids[0]
    res = run_training(o)
    print(json.dumps({k: res[k] for k in ("best_checkpoint", "best_is_ema", "best_regular_metric", "last_epoch")}))
    return 0


def _live(a) -> int:
    from ..live import FrameAnalyzer, SyntheticFrameSource, run_live
    pred, info = _predictor(a)
    src = SyntheticFrameSource(a.width, a.height, frames=a.frames)
    an = FrameAnalyzer(pred, [], threshold=a.threshold)
    st = run_live(src, an, out_dir=a.output, save_every=a.save_every)
    print(json.dumps({"preset_name": info["preset_name"], "frames_in": st.frames_in,
                      "frames_analyzed": st.frames_analyzed, "dropped": st.dropped, "fps": st.fps,
                      "latency_ms_p50": st.latency_ms_p50}))
    return 0


def _latency(a) -> int:
    ids = [int(x) for x in a.device_ids.split(",") if x.strip()] if a.device_ids else []
    if len(ids) > 1:
        return _latency_replicas(a, ids)
    pred, info = _predictor(a)
    r = pred.latency(a.iters, 20, a.batch_size, pin_cpus=not a.no_pin_cpus)
    print(json.dumps({"preset_name": info["preset_name"], **r}))
    return 0


def _latency_worker(rank, a, ids, barrier, queue):
    import torch
    a.device_id = ids[rank]
    torch.cuda.set_device(a.device_id)
    pred, info = _predictor(a)
    pred.latency(5, 20, a.batch_size, pin_cpus=not a.no_pin_cpus)   # capture and warm-up before the start
    barrier.wait()
    r = pred.latency(a.iters, 5, a.batch_size, pin_cpus=not a.no_pin_cpus)
    queue.put((rank, info["preset_name"], r))


def _latency_replicas(a, ids) -> int:
    """Data-parallel inference throughput: one model replica per GPU, one process each, all timed
    concurrently; reports the per-replica latencies and the summed images/s."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    barrier, queue = ctx.Barrier(len(ids)), ctx.Queue()
    procs = [ctx.Process(target=_latency_worker, args=(r, a, ids, barrier, queue)) for r in range(len(ids))]
    for p in procs:
        p.start()
    results = [queue.get(timeout=900) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    results.sort()
    per = [r for _, _, r in results]
    print(json.dumps({"preset_name": results[0][1], "replicas": len(ids), "batch": a.batch_size,
                      "images_per_s_total": round(sum(r["images_per_s"] for r in per), 1),
                      "p50_ms_max": round(max(r["p50_ms"] for r in per), 4),
                      "p99_ms_max": round(max(r["p99_ms"] for r in per), 4), "per_replica": per}))
    return 0 if all(p.exitcode == 0 for p in procs) else 1


def run(argv: Optional[List[str]] = None) -> int:
    a = build_parser().parse_args(argv)
    a.raw_argv = list(argv) if argv is not None else sys.argv[1:]
    logging.basicConfig(level=getattr(logging, str(a.log_level).upper(), logging.INFO),
                        filename=a.log_file or None, format="%(asctime)s %(levelname)s %(name)s: %(message)s")
    if a.cmd == "compile":
        return _compile(a)
    if a.cmd == "info":
        return _info(a.path)
    if a.cmd == "bench":
        return _bench(a)
    if a.cmd == "models":
        return _models()
    r = a.rcmd
    if r == "compile":
        return _compile(a)
    if r == "info":
        return _info(a.path)
    if r == "train":
        return _train(a)
    if r == "predict":
        return _predict(a)
    if r == "evaluate":
        return _evaluate(a)
    if r == "export-onnx":
        return _export(a)
    if r == "normalize-weights":
        from ..ckpt import normalize_checkpoint
        ck = normalize_checkpoint(a.input, a.output)
        print(json.dumps({"output": a.output, "tensors": len(ck.state_dict), "preset_name": ck.metadata.preset_name}))
        return 0
    if r == "build-engine":
        raise Unavailable("TensorRT is not installed in this environment; build-engine is unavailable")
    if r == "validate":
        return _validate(a)
    if r == "latency":
        return _latency(a)
    if r == "live":
        return _live(a)
    raise SystemExit(f"unknown command {r}")


def main(argv: Optional[List[str]] = None) -> int:
    try:
        return run(argv)
    except Unavailable as e:
        print(f"mmltk: unavailable: {e}", file=sys.stderr)
        return 2


if __name__ == "__main__":
    sys.exit(main())
