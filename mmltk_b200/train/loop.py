"""``run_training``: the epoch loop around :class:`TrainEngine`.

Reference: `src/rfdetr/training/train.cpp:1870-2730` -- option validation,
distributed context, loaders (rank-sharded, ``drop_last``), artifact
resolution with ``num_classes`` from the dataset, weights / resume, the epoch
loop, per-epoch validation of the regular and (optionally) EMA weights,
checkpoints (``checkpoint.pt`` for resume, ``checkpoint_epoch_<n>.pt``,
``checkpoint_best_regular.pt``, ``checkpoint_best_ema.pt``), ``progress.json``
(throttled, atomic), ``log.txt`` (one JSON line per epoch) and
``results.json``.

Differences by design:
* augmentation and target building run through :class:`GpuAugmenter`
  (host plan + one fused kernel), and the step through the CUDA-graph engine
  with the fused NVSwitch gradient step when more than one GPU is used;
* validation is distributed: every rank evaluates a shard of the validation
  split and the match records are all-gathered, instead of rank 0 alone.
"""
from __future__ import annotations

import json
import logging
import math
import os
import threading
import time
from typing import Dict, Optional

import torch

from ..ckpt import CheckpointMetadata, load_native_checkpoint, save_native_checkpoint
from ..ckpt.native import state_from_archive, state_to_archive
from ..ops._ext import native
from ..config import TrainOptions
from ..data.augment import GpuAugmenter
from ..data.loader import BatchLoader, CompiledDataset
from ..infer.predictor import Predictor, resolve_model
from ..parallel.launch import DistContext, init_distributed
from ..utils.runtime import setup_host_runtime

__all__ = ["run_training", "ProgressWriter", "checkpoint_metric", "evaluate", "validation_loss"]

log = logging.getLogger("mmltk.train")


class ProgressWriter:
    """Latest-state JSON file: throttled writes, atomic replace, ``phase: "error"`` on failure
    (reference `LatestJsonWriter`, `train.cpp:606-768`)."""

    def __init__(self, path: str, min_interval_s: float = 0.25):
        self.path = path
        self.min_interval = min_interval_s
        self.last = 0.0
        self.state: Dict = {}
        self.lock = threading.Lock()

    def submit(self, update: Dict, force: bool = False) -> None:
        with self.lock:
            self.state.update(update)
            now = time.monotonic()
            if not force and now - self.last < self.min_interval:
                return
            self.last = now
            tmp = self.path + ".tmp"
            with open(tmp, "w") as f:
                json.dump(self.state, f, indent=1)
            os.replace(tmp, self.path)

    def error(self, message: str) -> None:
        self.submit({"phase": "error", "error": message}, force=True)


def _validation_record(opts, paths, ctx, epoch: int, source: str, summary: Dict, seconds: float) -> None:
    """``--validation-profile``: one JSON line per validation pass (reference
    `validation_profile.jsonl`, `src/rfdetr/inference/evaluator.cpp:1490-1560`)."""
    if not (opts.validation_profile and ctx.main):
        return
    rec = {"event": "rfdetr.validation.pass", "event_source": "train", "epoch": epoch, "validation_pass": epoch,
           "model_source": source, "world_size": ctx.world_size, "total_wall_seconds": seconds,
           "metric_mode": "bbox_and_mask" if "segm" in summary else "bbox", **_summary_json(summary),
           "val_loss": summary.get("loss")}
    with open(os.path.join(os.path.dirname(paths["log"]), "validation_profile.jsonl"), "a") as f:
        f.write(json.dumps(rec) + "\n")


def checkpoint_metric(summary: Dict, masks: bool) -> float:
    key = "segm" if masks and "segm" in summary else "bbox"
    return float(summary[key]["ap"])


def _summary_json(s: Optional[Dict]) -> Dict:
    if not s:
        return {}
    out = {"bbox": {k: s["bbox"][k] for k in ("ap", "ap50", "ap75")}}
    if "segm" in s:
        out["mask"] = {k: s["segm"][k] for k in ("ap", "ap50", "ap75")}
    return out


def _augmentation_json(a) -> Dict:
    g = lambda x: {"probability": x.probability, "min_strength": x.min_strength, "max_strength": x.max_strength}
    return {"enabled": a.enabled, "geometry": g(a.geometry), "resize": g(a.resize), "color": g(a.color),
            "noise": g(a.noise), "blur": g(a.blur), "occlusion": g(a.occlusion),
            "copy_paste_probability": a.copy_paste_probability}


def _resume_extra(opts: TrainOptions, engine, epoch: int, best_regular: float, best_ema: float) -> Dict:
    d = {"optimizer_kind": opts.optimizer, "optimizer": engine.optimizer_state(), "epoch": int(epoch),
         "lr_scheduler": opts.lr_scheduler, "lr_drop": int(opts.lr_drop), "warmup_epochs": float(opts.warmup_epochs),
         "warmup_momentum": float(opts.warmup_momentum), "lr_min_factor": float(opts.lr_min_factor),
         "gpu_augment_enabled": bool(opts.augmentation.enabled), "best_regular_metric": float(best_regular),
         "best_ema_metric": float(best_ema), "grad_scaler_scale": 1.0, "grad_scaler_growth_tracker": 0}
    a = opts.augmentation
    for name in ("geometry", "resize", "color", "noise", "blur", "occlusion"):
        g = getattr(a, name)
        d[f"gpu_augment_{name}_probability"] = float(g.probability)
        d[f"gpu_augment_{name}_min_strength"] = float(g.min_strength)
        d[f"gpu_augment_{name}_max_strength"] = float(g.max_strength)
    d["gpu_augment_copy_paste_probability"] = float(a.copy_paste_probability)
    ema = engine.ema_state()
    if ema is not None:
        d["ema_state"] = state_to_archive({k: v.float().cpu() for k, v in ema.items()})
    return d


def _check_resume(extra: Dict, opts: TrainOptions) -> None:
    for key, cur in (("lr_scheduler", opts.lr_scheduler), ("lr_drop", opts.lr_drop),
                     ("warmup_epochs", opts.warmup_epochs), ("warmup_momentum", opts.warmup_momentum),
                     ("lr_min_factor", opts.lr_min_factor)):
        if key in extra and extra[key] != cur:
            raise ValueError(f"resume checkpoint {key} ({extra[key]!r}) does not match the current options ({cur!r})")
    if extra.get("optimizer_kind", "adamw") != opts.optimizer:
        raise ValueError("resume checkpoint optimizer_kind does not match the current options")
    if "optimizer" not in extra:
        raise ValueError("resume checkpoint is missing the optimizer state")


def evaluate(model_fp32: torch.nn.Module, compiled: str, ctx: DistContext, batch_size: int, max_dets: int,
             masks: bool, shard: bool = True, with_loss: bool = False, sample_png: Optional[str] = None,
             gather=None) -> Dict:
    """COCO AP of a model over a compiled split; each rank takes every world-th batch.
    ``sample_png``: the main rank also writes its first validation image with the predictions drawn
    on the GPU (reference: the eval sample image of `train.cpp:158-265`)."""
    from ..eval import CocoEvaluator
    pred = Predictor(model_fp32, device=ctx.device, cuda_graph=ctx.device.type == "cuda", with_masks=masks)
    ev = CocoEvaluator(compiled, masks=masks, max_dets=max_dets)
    bl = BatchLoader(compiled, batch_size, shuffle=False, pixels="uint8", max_targets=1,
                     shard_rank=ctx.rank if shard else 0, shard_count=ctx.world_size if shard else 1,
                     device=ctx.device if ctx.device.type == "cuda" else None)
    for images, _t, idx in bl:
        if images.shape[0] != batch_size and pred.use_graph:
            pad = torch.zeros(batch_size - images.shape[0], *images.shape[1:], dtype=images.dtype,
                              device=images.device)
            res = {k: v[:len(idx)] for k, v in pred(torch.cat([images, pad])).items()}
        else:
            res = pred(images)
        ev.add(idx, res["scores"], res["labels"], res["boxes"], res.get("masks"))
        if sample_png and ctx.main:
            _write_eval_sample(images[0], {k: v[:1] for k, v in res.items()}, bl.dataset.class_names, sample_png)
            sample_png = None
    # images left over by the per-rank sharding (fewer than one batch per rank) go to rank 0
    n = len(bl.dataset)
    covered = len(bl) * batch_size * (ctx.world_size if shard else 1)
    if ctx.main and covered < n:
        rest = list(range(covered, n))
        for s in range(0, len(rest), batch_size):
            ids = rest[s:s + batch_size]
            x = torch.stack([(bl.dataset.image(i) * 255).round().to(torch.uint8) for i in ids]).to(ctx.device)
            res = pred._step(x)
            ev.add(ids, res["scores"], res["labels"], res["boxes"], res.get("masks"))
    pred.release()
    if shard and ctx.enabled:
        ev.reduce(gather=gather)
    out = ev.summarize()
    if with_loss:
        out["loss"] = validation_loss(pred.model, compiled, ctx, batch_size, shard)
    return out


def _write_eval_sample(image_u8, res, class_names, path: str, threshold: float = 0.3) -> None:
    from ..infer.visualize import draw_detections
    os.makedirs(os.path.dirname(path) or ".", exist_ok=True)
    hwc = image_u8.permute(1, 2, 0).contiguous()
    hwc = draw_detections(hwc, {k: v[0] for k, v in res.items()}, class_names, threshold)
    with open(path, "wb") as f:
        f.write(native().encode_png(hwc.cpu()))


@torch.no_grad()
def validation_loss(model, compiled: str, ctx: DistContext, batch_size: int, shard: bool = True) -> float:
    """Mean weighted criterion loss over a compiled split, eval-mode outputs (one query group),
    averaged across ranks (reference `--validation-loss`, `train.cpp:1513-1868`)."""
    from ..criterion import SetCriterion
    from ..data.augment import normalize_images
    ds = CompiledDataset(compiled)
    counts = ds.reader.instance_counts()
    slots = max(1, int(counts.max()) if counts.numel() else 1)
    crit = SetCriterion(model.cfg)
    dev = ctx.device
    bl = BatchLoader(compiled, batch_size, shuffle=False, pixels="uint8", max_targets=slots,
                     shard_rank=ctx.rank if shard else 0, shard_count=ctx.world_size if shard else 1,
                     device=dev if dev.type == "cuda" else None)
    was_training = model.training
    model.eval()
    dtype = next(model.parameters()).dtype
    total = torch.zeros((), dtype=torch.float64, device=dev)
    n = torch.zeros((), dtype=torch.float64, device=dev)
    for images, targets, idx in bl:
        x = normalize_images(images.to(dev), dtype if dev.type == "cuda" else torch.float32)
        out = model(x, include_masks=bool(model.cfg.segmentation))
        losses, _ = crit(out, targets.to(dev), training=False)
        total += crit.weighted(losses).double() * len(idx)
        n += len(idx)
    if ctx.enabled:
        import torch.distributed as dist
        both = torch.stack([total, n]).to(dev)
        dist.all_reduce(both)
        total, n = both[0], both[1]
    model.train(was_training)
    return float(total / n.clamp(min=1))


def run_training(opts: TrainOptions, ctx: Optional[DistContext] = None) -> Dict:
    opts.validate()
    if not opts.train_compiled or not opts.val_compiled or not opts.output_dir:
        raise ValueError("train needs --train-compiled, --val-compiled and --output-dir")
    if bool(opts.weights) == bool(opts.resume) and (opts.weights or opts.resume):
        raise ValueError("pass exactly one of --weights / --resume")
    own_ctx = ctx is None
    if ctx is None:
        ctx = init_distributed(opts.dist_rank if opts.dist_worker else None,
                               opts.dist_world_size if opts.dist_worker else None, opts.device_id,
                               opts.dist_store_file)
    torch.manual_seed(opts.seed + ctx.rank)
    out_dir = opts.output_dir
    paths = {k: os.path.join(out_dir, v) for k, v in dict(
        progress="progress.json", log="log.txt", results="results.json", ckpt="checkpoint.pt",
        best_regular="checkpoint_best_regular.pt", best_ema="checkpoint_best_ema.pt").items()}
    progress = None
    if ctx.main:
        os.makedirs(out_dir, exist_ok=True)
        for k in ("progress", "log", "results"):
            if os.path.exists(paths[k]):
                os.remove(paths[k])
        progress = ProgressWriter(paths["progress"])
    try:
        result = _train(opts, ctx, paths, progress)
    except BaseException as e:
        if progress is not None:
            progress.error(f"{type(e).__name__}: {e}")
        raise
    finally:
        if own_ctx:
            ctx.close()
    return result


def _train(opts: TrainOptions, ctx: DistContext, paths: Dict[str, str], progress: Optional[ProgressWriter]) -> Dict:
    from .engine import TrainEngine
    train_ds = CompiledDataset(opts.train_compiled)
    W, H = train_ds.size
    if W != H:
        raise ValueError(f"compiled train images must be square (got {W}x{H})")
    if opts.resolution and opts.resolution != W:
        raise ValueError(f"--resolution {opts.resolution} differs from the compiled image size {W}")
    num_classes = train_ds.num_classes
    resume = load_native_checkpoint(opts.resume) if opts.resume else None
    if resume is not None:
        _check_resume(resume.extra, opts)
    model, info = resolve_model(opts.weights or opts.resume or None, preset=opts.preset or None, resolution=W,
                                num_classes=num_classes, strict=False)
    cfg = model.cfg
    masks = bool(cfg.segmentation)
    counts = train_ds.reader.instance_counts()
    slots = int(counts.max()) + 1 if counts.numel() else 1
    slots = max(1, min(slots, 256))
    rt = setup_host_runtime(opts.workers, 1, max(2, opts.prefetch_factor), opts.cpu_affinity,
                            pin=ctx.device.type == "cuda", high_priority=opts.high_priority)
    if ctx.main:
        log.info("host runtime: %s", rt.describe())
        log.info("training: torch %s, bf16, optimizer %s, gradient step %s, cuda graph %s, world %d, "
                 "batch %d per rank x %d accumulation = %d per rank, %d global", torch.__version__,
                 opts.optimizer, ("fused-nvswitch" if opts.ddp_backend == "fused" and opts.optimizer == "adamw"
                                  else "nccl") if ctx.enabled else "single-gpu",
                 opts.cuda_graph and ctx.device.type == "cuda", ctx.world_size, opts.batch_size,
                 opts.micro_batches_per_step(), opts.batch_size * opts.micro_batches_per_step(),
                 opts.batch_size * opts.micro_batches_per_step() * ctx.world_size)
    loader = BatchLoader(opts.train_compiled, opts.batch_size, shuffle=True, seed=opts.seed, shard_rank=ctx.rank,
                         shard_count=ctx.world_size, drop_last=True, pixels="uint8", workers=max(1, rt.split["gather"]),
                         prefetch=max(2, opts.prefetch_factor), max_targets=1,
                         device=ctx.device if ctx.device.type == "cuda" else None,
                         cpus=rt.loader_cpus[:1] if ctx.device.type == "cuda" else None)
    batches = len(loader)
    micro = opts.micro_batches_per_step()       # --grad-accum-steps x --lanes batches per optimizer step
    steps_per_epoch = batches // micro
    if steps_per_epoch == 0:
        raise ValueError("the compiled train split is too small for one effective batch per rank; reduce "
                         "--batch-size, --grad-accum-steps or the world size")
    total_steps = max(1, steps_per_epoch * opts.epochs)
    grad_sync = None
    if ctx.enabled:
        if ctx.device.type == "cuda" and opts.ddp_backend == "fused":
            from ..parallel.fused import FusedGradSync
            grad_sync = FusedGradSync()
        else:
            from ..parallel.ddp import NcclGradSync
            grad_sync = NcclGradSync()
    # evaluation's match-record all-gather: over peer memory when the fused NVSwitch sync is in use
    gather = getattr(grad_sync, "all_gather_tensor", None)
    engine = TrainEngine(model, opts, ctx.device, grad_sync, max_targets=slots, steps_per_epoch=steps_per_epoch,
                         total_steps=total_steps)
    if ctx.device.type == "cuda":
        engine.bind_static_inputs(opts.batch_size, 3, H, W)
    start_epoch, best_regular, best_ema = 0, -math.inf, -math.inf
    if resume is not None:
        engine.load_optimizer_state(resume.extra["optimizer"])
        if "ema_state" in resume.extra:
            engine.load_ema_state(state_from_archive(resume.extra["ema_state"]))
        start_epoch = int(resume.extra.get("epoch", -1)) + 1
        best_regular = float(resume.extra.get("best_regular_metric", -math.inf))
        best_ema = float(resume.extra.get("best_ema_metric", -math.inf))
    augmenter = GpuAugmenter(opts.augmentation, opts.batch_size, H, W, slots, device=ctx.device, masks=masks,
                             seed=opts.seed, rank=ctx.rank)
    meta = CheckpointMetadata.from_config(cfg, "native", info.get("weights_path", ""))
    val_bs = opts.val_batch_size or opts.batch_size
    best_path, best_is_ema = None, False
    if ctx.main:
        if math.isfinite(best_regular) and os.path.exists(paths["best_regular"]):
            best_path = paths["best_regular"]
        if math.isfinite(best_ema) and os.path.exists(paths["best_ema"]) and best_ema >= best_regular:
            best_path, best_is_ema = paths["best_ema"], True
        progress.submit({"phase": "starting", "epoch": start_epoch, "total_epochs": opts.epochs,
                         "completed_batches": 0, "total_batches": batches, "optimizer_steps": 0,
                         "steps_per_epoch": steps_per_epoch, "train_loss": 0.0, "step_loss": 0.0,
                         "batches_per_second": 0.0, "images_per_second": 0.0, "elapsed_seconds": 0.0,
                         "checkpoint_path": "", "val_loss": None, "val": {}}, force=True)
    history = []
    t_start = time.monotonic()
    seq = 0
    last_epoch = start_epoch - 1
    for epoch in range(start_epoch, opts.epochs):
        loader.set_epoch(epoch)
        loss_sum, n_loss, t_epoch = 0.0, 0, time.monotonic()

        def consume(b, pending):
            # read step b's loss once it has finished; the next batch was queued meanwhile
            nonlocal loss_sum, n_loss
            r = pending.result()
            if r.grad_norm is not None or not ctx.device.type == "cuda":
                loss_sum += float(r.loss)
                n_loss += 1
            if ctx.main and opts.print_freq > 0 and (b + 1) % opts.print_freq == 0:
                el = time.monotonic() - t_epoch
                log.info("epoch %d step %d/%d loss %.4f (mean %.4f) grad_norm %s %.1f img/s", epoch, b + 1,
                         steps_per_epoch * micro, float(r.loss), loss_sum / max(1, n_loss),
                         "-" if r.grad_norm is None else f"{r.grad_norm:.3f}",
                         (b + 1) * opts.batch_size * ctx.world_size / max(el, 1e-9))
            if progress is not None:
                el = time.monotonic() - t_epoch
                progress.submit({"phase": "train", "epoch": epoch, "completed_batches": b + 1,
                                 "optimizer_steps": engine.step_count, "train_loss": loss_sum / max(1, n_loss),
                                 "step_loss": float(r.loss), "batches_per_second": (b + 1) / max(el, 1e-9),
                                 "images_per_second": (b + 1) * opts.batch_size * ctx.world_size / max(el, 1e-9),
                                 "elapsed_seconds": time.monotonic() - t_start})

        prev = None
        for b, (images, _plain, idx) in enumerate(loader):
            if b >= steps_per_epoch * micro:
                break
            st = augmenter.prepare(idx, loader.dataset.reader, epoch, seq)
            seq += 1
            x, targets = augmenter.apply(images, st)
            pending = engine.step_async(x, targets)
            if prev is not None:
                consume(*prev)
            prev = (b, pending)
        if prev is not None:
            consume(*prev)
        train_loss = loss_sum / max(1, n_loss)
        # validation: regular weights, then EMA
        if progress is not None:
            progress.submit({"phase": "validate", "epoch": epoch}, force=True)
        regular = engine.export_model("master")
        t_val = time.monotonic()
        val = evaluate(regular, opts.val_compiled, ctx, val_bs, opts.eval_max_dets, masks,
                       with_loss=opts.validation_loss,
                       sample_png=os.path.join(opts.output_dir, "eval_samples", f"epoch_{epoch:04d}.png"),
                       gather=gather)
        _validation_record(opts, paths, ctx, epoch, "regular", val, time.monotonic() - t_val)
        ema_val = None
        ema_model = engine.export_model("ema") if opts.use_ema else None
        if ema_model is not None:
            t_val = time.monotonic()
            ema_val = evaluate(ema_model, opts.val_compiled, ctx, val_bs, opts.eval_max_dets, masks,
                               with_loss=opts.validation_loss, gather=gather)
            _validation_record(opts, paths, ctx, epoch, "ema", ema_val, time.monotonic() - t_val)
        if ctx.main:
            state = regular.state_dict()
            save_native_checkpoint(os.path.join(os.path.dirname(paths["ckpt"]), f"checkpoint_epoch_{epoch + 1}.pt"),
                                   state, meta)
            m = checkpoint_metric(val, masks)
            if m > best_regular:
                best_regular = m
                save_native_checkpoint(paths["best_regular"], state, meta)
                best_path, best_is_ema = paths["best_regular"], False
            if ema_val is not None:
                me = checkpoint_metric(ema_val, masks)
                if me > best_ema:
                    best_ema = me
                    save_native_checkpoint(paths["best_ema"], ema_model.state_dict(), meta)
                    best_path, best_is_ema = paths["best_ema"], True
        extra = _resume_extra(opts, engine, epoch, best_regular, best_ema)   # collective when sharded
        if ctx.main:
            save_native_checkpoint(paths["ckpt"], regular.state_dict(), meta, extra)
            rec = {"epoch": epoch, "train_lanes": max(1, opts.lanes), "eval_lanes": 1,
                   "effective_batch_per_rank": opts.batch_size * micro,
                   "effective_batch_global": opts.batch_size * micro * ctx.world_size,
                   "train_loss": train_loss, "val_loss": val.get("loss"), "val": _summary_json(val),
                   "ema_val_loss": None if ema_val is None else ema_val.get("loss"),
                   "ema_val": _summary_json(ema_val)}
            with open(paths["log"], "a") as f:
                f.write(json.dumps(rec) + "\n")
            history.append(rec)
            progress.submit({"phase": "epoch_complete", "epoch": epoch, "val": _summary_json(val),
                             "checkpoint_path": best_path or paths["ckpt"]}, force=True)
        last_epoch = epoch
        ctx.barrier()
    engine.release_graph()
    result = {"preset_name": cfg.preset_name, "output_dir": opts.output_dir, "checkpoint": paths["ckpt"],
              "best_checkpoint": best_path or paths["ckpt"], "best_is_ema": best_is_ema,
              "best_regular_metric": best_regular, "best_ema_metric": best_ema, "last_epoch": last_epoch,
              "history_size": len(history), "train_lanes": max(1, opts.lanes), "eval_lanes": 1,
              "effective_batch_per_rank": opts.batch_size * micro,
              "effective_batch_global": opts.batch_size * micro * ctx.world_size,
              "gpu_augmentation": _augmentation_json(opts.augmentation), "test": {}}
    if opts.test_compiled:
        best = resolve_model(result["best_checkpoint"], preset=cfg.preset_name, num_classes=num_classes,
                             strict=False)[0]
        result["test"] = _summary_json(evaluate(best, opts.test_compiled, ctx, val_bs, opts.eval_max_dets, masks,
                                                gather=gather))
    if ctx.main:
        with open(paths["results"], "w") as f:
            json.dump(result, f, indent=1)
        progress.submit({"phase": "complete"}, force=True)
    if grad_sync is not None and hasattr(grad_sync, "close"):
        ctx.barrier()
        grad_sync.close()
    return result
