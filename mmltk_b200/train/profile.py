"""Kernel-time breakdown of one training step (``torch.profiler``, CUDA activity).

    python -m mmltk_b200.train.profile --preset rf-detr-medium --batch-size 8 --steps 2

Runs warm-up steps, then profiles ``--steps`` eager steps of the same engine the
bench uses (eager, so every kernel is attributed; the bench replays the
captured graph) and prints a markdown table of CUDA time per kernel, grouped
by kernel name, plus the graph-replay step time measured with CUDA events.
"""
from __future__ import annotations

import argparse
import collections
import sys

import torch


def _origin(ev, stack: bool = False) -> str:
    """Nearest enclosing autograd node (backward) or autograd Function / module-level op (forward);
    with ``stack``, forward ops outside an autograd Function name their innermost frame in this package."""
    if stack and ev.stack:
        for fr in ev.stack:
            if "mmltk_b200" in fr and "profile.py" not in fr:
                return fr.split("mmltk_b200/")[-1]
    p = ev.cpu_parent
    while p is not None:
        n = p.name
        if n.startswith("autograd::engine::evaluate_function: "):
            return n.split(": ", 1)[1]
        if not n.startswith("aten::") and not n.startswith("cuda") and not n.startswith("ProfilerStep"):
            return n
        p = p.cpu_parent
    return "-"


def origin_table(events, steps: int, top: int, shapes: bool = False, stack: bool = False) -> str:
    """CUDA time of each aten op's own kernels, keyed by (op, origin[, input shapes])."""
    per = collections.Counter()
    count = collections.Counter()
    for ev in events:
        if ev.device_type != torch.autograd.DeviceType.CPU or not ev.name.startswith("aten::"):
            continue
        t = sum(k.duration for k in ev.kernels)
        if not ev.kernels:
            continue
        org = _origin(ev, stack)
        if shapes:
            org = f"{org} {str(ev.input_shapes)[:70]}"
        key = (ev.name, org)
        per[key] += t
        count[key] += len(ev.kernels)
    total = sum(per.values()) or 1.0
    lines = ["| share | ms/step | kernels/step | aten op | origin |", "|---|---|---|---|---|"]
    for (name, org), t in per.most_common(top):
        lines.append(f"| {100 * t / total:.1f}% | {t / 1e3 / steps:.3f} | {count[(name, org)] // steps} | "
                     f"`{name}` | `{org[:150]}` |")
    return "\n".join(lines)


def _kernel_table(events, steps: int, top: int) -> str:
    per = collections.Counter()
    count = collections.Counter()
    for ev in events:
        if ev.device_type == torch.autograd.DeviceType.CUDA:
            per[ev.name] += ev.device_time
            count[ev.name] += 1
    total = sum(per.values()) or 1.0
    lines = [f"CUDA time {total / 1e3 / steps:.3f} ms/step over {steps} eager steps "
             f"({sum(count.values()) // steps} kernels/step)\n",
             "| share | ms/step | launches/step | kernel |", "|---|---|---|---|"]
    for name, t in per.most_common(top):
        lines.append(f"| {100 * t / total:.1f}% | {t / 1e3 / steps:.4f} | {count[name] // steps} | `{name[:110]}` |")
    return "\n".join(lines)


def _profile_infer(a) -> int:
    """Eager forward of the inference Predictor (kernel table), then its CUDA-graph latency."""
    from torch.profiler import ProfilerActivity, profile

    from ..infer import Predictor
    from ..models.rfdetr import build_model
    torch.manual_seed(0)
    model = build_model(a.preset).eval()
    dev = torch.device("cuda", 0)
    pred = Predictor(model, device=dev, cuda_graph=False)
    x = torch.randint(0, 256, (a.batch_size, 3, *pred.size), dtype=torch.uint8, device=dev)
    for _ in range(a.warmup):
        pred(x)
    torch.cuda.synchronize()
    acts = [ProfilerActivity.CPU, ProfilerActivity.CUDA] if a.by_origin else [ProfilerActivity.CUDA]
    with profile(activities=acts, record_shapes=a.by_origin and not a.no_shapes,
                 with_stack=a.by_origin and a.stack) as prof:
        for _ in range(a.steps):
            pred(x)
        torch.cuda.synchronize()
    print(f"# {a.preset} inference, batch {a.batch_size}, {pred.size[0]}x{pred.size[1]}, bf16\n")
    if a.by_origin:
        print(origin_table(prof.events(), a.steps, a.top, shapes=not a.no_shapes, stack=a.stack))
    else:
        print(_kernel_table(prof.events(), a.steps, a.top))
    g = Predictor(model, device=dev, cuda_graph=True)
    print(f"\nCUDA-graph latency: {g.latency(200, 20, a.batch_size)}")
    return 0


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--preset", default="rf-detr-medium")
    ap.add_argument("--batch-size", type=int, default=8)
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--top", type=int, default=30)
    ap.add_argument("--by-op", action="store_true", help="rank aten ops (with input shapes) instead of kernels")
    ap.add_argument("--no-shapes", action="store_true", help="with --by-op / --by-origin: leave input shapes out")
    ap.add_argument("--by-origin", action="store_true",
                    help="rank (aten op, enclosing autograd node or autograd Function) pairs by CUDA time")
    ap.add_argument("--stack", action="store_true", help="with --by-origin: name forward ops by source line")
    ap.add_argument("--infer", action="store_true",
                    help="profile the inference Predictor (eval model, uint8 input -> top-k results) instead")
    a = ap.parse_args(argv)
    if not torch.cuda.is_available():
        print("profile: needs a GPU", file=sys.stderr)
        return 2
    if a.infer:
        return _profile_infer(a)
    from ..config import TrainOptions
    from ..data.synthetic import synthetic_batch
    from ..models.rfdetr import build_model
    from .engine import TrainEngine
    torch.manual_seed(0)
    model = build_model(a.preset)
    cfg = model.cfg
    opts = TrainOptions(batch_size=a.batch_size, use_ema=True, cuda_graph=False)
    dev = torch.device("cuda", 0)
    images, targets = synthetic_batch(a.batch_size, cfg.resolution, seed=0, kmax=10, slots=10, dtype=torch.bfloat16)
    images, targets = images.to(dev), targets.to(dev)
    eng = TrainEngine(model, opts, dev, max_targets=targets.slots, steps_per_epoch=1000, total_steps=1000)
    eng.bind_static_inputs(a.batch_size, 3, cfg.resolution, cfg.resolution)
    for _ in range(a.warmup):
        eng.step(images, targets)
    torch.cuda.synchronize()
    from torch.profiler import ProfilerActivity, profile
    if a.by_origin:
        with profile(activities=[ProfilerActivity.CPU, ProfilerActivity.CUDA], record_shapes=not a.no_shapes,
                     with_stack=a.stack) as prof:
            for _ in range(a.steps):
                eng.step()
            torch.cuda.synchronize()
        print(origin_table(prof.events(), a.steps, a.top, shapes=not a.no_shapes, stack=a.stack))
        return 0
    if a.by_op:
        # aten ops with input shapes, ranked by the CUDA time of the kernels they launched
        with profile(activities=[ProfilerActivity.CPU, ProfilerActivity.CUDA], record_shapes=True) as prof:
            for _ in range(a.steps):
                eng.step()
            torch.cuda.synchronize()
        print(prof.key_averages(group_by_input_shape=not a.no_shapes).table(
            sort_by="self_cuda_time_total", row_limit=a.top, max_name_column_width=60, max_shapes_column_width=90))
        return 0
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(a.steps):
            eng.step()
        torch.cuda.synchronize()
    per = collections.Counter()
    count = collections.Counter()
    for ev in prof.events():
        if ev.device_type == torch.autograd.DeviceType.CUDA:
            per[ev.name] += ev.device_time
            count[ev.name] += 1
    total = sum(per.values())
    print(f"# {a.preset} train step, batch {a.batch_size}, {cfg.resolution}x{cfg.resolution}, bf16\n")
    print(f"CUDA time {total / 1e3 / a.steps:.2f} ms/step over {a.steps} eager steps "
          f"({sum(count.values()) // a.steps} kernels/step)\n")
    print("| share | ms/step | launches/step | kernel |\n|---|---|---|---|")
    for name, t in per.most_common(a.top):
        print(f"| {100 * t / total:.1f}% | {t / 1e3 / a.steps:.3f} | {count[name] // a.steps} | "
              f"`{name[:110]}` |")
    # graph replay for comparison
    opts.cuda_graph = True
    eng2 = eng
    eng2.opts.cuda_graph = True
    for _ in range(4):
        eng2.step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(10):
        eng2.step(sync=False)
    e1.record()
    e1.synchronize()
    print(f"\nCUDA-graph replay: {e0.elapsed_time(e1) / 10:.3f} ms/step "
          f"({a.batch_size * 10000 / e0.elapsed_time(e1):.1f} img/s)")
    eng2.release_graph()
    return 0


if __name__ == "__main__":
    sys.exit(main())
