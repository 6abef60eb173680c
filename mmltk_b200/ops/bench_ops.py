"""Kernel micro-benchmarks: the framework's sm_100a kernels against the
library baseline of the same op, timed with CUDA events after warm-up.

    python -m mmltk_b200.ops.bench_ops gemm      # tcgen05 GEMM vs cuBLAS on the RF-DETR-M shapes
    python -m mmltk_b200.ops.bench_ops msda      # MSDeformAttn fwd+bwd vs fp32 reference path
    python -m mmltk_b200.ops.bench_ops attn      # attention fwd+bwd of the RF-DETR-M shapes per SDPA backend
    python -m mmltk_b200.ops.bench_ops kernels   # LayerNorm, criterion (matcher + solver + losses), post-process

Inputs are larger than L2 where the op allows; each timing is the median of
several event-timed runs.
"""
from __future__ import annotations

import argparse
import json
import statistics

import torch

__all__ = ["time_ms", "time_graph_ms", "bench_gemm", "bench_msda", "bench_attn"]


def time_ms(fn, warmup: int = 5, iters: int = 20, reps: int = 5) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    out = []
    for _ in range(reps):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(iters):
            fn()
        e.record()
        torch.cuda.synchronize()
        out.append(s.elapsed_time(e) / iters)
    return statistics.median(out)


def time_graph_ms(fn, iters: int = 20, reps: int = 5) -> float:
    """Device time per call of ``fn`` with the host out of the loop: ``iters`` calls are
    captured in one CUDA graph and the replays are event-timed (median of ``reps``)."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(iters):
            fn()
    return time_ms(g.replay, warmup=2, iters=1, reps=reps) / iters


# (name, M, N, K, mode): mode nt = x W^T, nn = dY W, tn = dY^T X
GEMM_SHAPES = [
    ("vit.qkv.fwd", 10400, 1152, 384, "nt"), ("vit.proj.fwd", 10400, 384, 384, "nt"),
    ("vit.fc1.fwd", 10400, 1536, 384, "nt"), ("vit.fc2.fwd", 10400, 384, 1536, "nt"),
    ("vit.fc1.dgrad", 10400, 384, 1536, "nn"), ("vit.fc2.dgrad", 10400, 1536, 384, "nn"),
    ("vit.fc1.wgrad", 1536, 384, 10400, "tn"), ("vit.fc2.wgrad", 384, 1536, 10400, "tn"),
    ("dec.ffn1.fwd", 31200, 2048, 256, "nt"), ("dec.ffn2.fwd", 31200, 256, 2048, "nt"),
    ("dec.ffn1.wgrad", 2048, 256, 31200, "tn"), ("dec.ffn2.dgrad", 31200, 2048, 256, "nn"),
    # the training forms: bias + GELU / ReLU epilogue that also stores the pre-activation
    ("vit.fc1.fwd.gelu_aux", 10400, 1536, 384, "nt_gelu"), ("dec.ffn1.fwd.relu_aux", 31200, 2048, 256, "nt_relu"),
    # main-loop probe: one 128 x 256 tile per SM (one 256 x 256 pair tile per two SMs), a long reduction
    ("probe.mainloop", 18944, 256, 8192, "nt"),
]


def bench_gemm(device="cuda", only=None, quick=False):
    from ._ext import kernels
    k = kernels()
    rows = []
    for name, M, N, K, mode in GEMM_SHAPES:
        if only and name != only:
            continue
        g = torch.Generator(device=device).manual_seed(0)
        if mode == "nt":
            a = torch.randn(M, K, device=device, generator=g).bfloat16()
            b = torch.randn(N, K, device=device, generator=g).bfloat16()
            ours = lambda: k.gemm_tc(a, b, None, False, False)  # noqa: E731
            lib = lambda: torch.mm(a, b.t())  # noqa: E731
        elif mode in ("nt_gelu", "nt_relu"):
            import torch.nn.functional as F
            a = torch.randn(M, K, device=device, generator=g).bfloat16()
            b = (torch.randn(N, K, device=device, generator=g) * K ** -0.5).bfloat16()
            bias = torch.randn(N, device=device, generator=g).bfloat16()
            epi, act = (1, F.gelu) if mode == "nt_gelu" else (2, F.relu)
            ours = lambda: k.gemm_tc(a, b, bias, False, False, epi, True)  # noqa: E731

            def lib():   # cuBLAS GEMM with bias epilogue, then the activation (pre kept for backward)
                pre = torch.addmm(bias, a, b.t())
                return act(pre), pre
        elif mode == "nn":
            a = torch.randn(M, K, device=device, generator=g).bfloat16()
            b = torch.randn(K, N, device=device, generator=g).bfloat16()
            ours = lambda: k.gemm_tc(a, b, None, False, True)  # noqa: E731
            lib = lambda: torch.mm(a, b)  # noqa: E731
        else:
            a = torch.randn(K, M, device=device, generator=g).bfloat16()
            b = torch.randn(K, N, device=device, generator=g).bfloat16()
            ours = lambda: k.gemm_tc(a, b, None, True, True)  # noqa: E731
            lib = lambda: torch.mm(a.t(), b)  # noqa: E731
        ref = lib()
        ref = (ref[0] if isinstance(ref, tuple) else ref).float()
        got = ours()[0].float()
        err = ((got - ref).abs().max() / ref.abs().max()).item()
        if quick:  # a few launches only (for profiler captures)
            for _ in range(3):
                ours()
            torch.cuda.synchronize()
            continue
        # device time from CUDA-graph replays, as in the training step (host launch cost excluded)
        t_ours, t_lib = time_graph_ms(ours), time_graph_ms(lib)
        fl = 2.0 * M * N * K
        row = {"shape": name, "M": M, "N": N, "K": K, "mode": mode, "ms_tc": round(t_ours, 4),
               "ms_cublas": round(t_lib, 4), "tflops_tc": round(fl / t_ours / 1e9, 1),
               "tflops_cublas": round(fl / t_lib / 1e9, 1), "speedup": round(t_lib / t_ours, 3),
               "rel_err": err}
        # the two tile variants forced: single-CTA 128-row tiles / CTA-pair 256-row tiles
        for v in (1, 2):
            k.gemm_tc_set_variant(v)
            try:
                e_v = ((ours()[0].float() - ref).abs().max() / ref.abs().max()).item()
                t_v = time_graph_ms(ours)
                row[f"ms_tc{v}"], row[f"tflops_tc{v}"], row[f"rel_err_tc{v}"] = round(t_v, 4), round(fl / t_v / 1e9, 1), e_v
            finally:
                k.gemm_tc_set_variant(0)
        row["status"] = k.gemm_tc_status(torch.cuda.current_device())
        rows.append(row)
    return rows


def bench_msda(device="cuda", quick=False):
    """value [16, 6480, 16, 16] bf16, Lq 3900, 2 levels (72x72, 36x36), 4 points."""
    from .msda import msda, msda_reference
    B, H, D, Lq, P = 16, 16, 16, 3900, 4
    shapes = [(72, 72), (36, 36)]
    S = sum(h * w for h, w in shapes)
    L = len(shapes)
    g = torch.Generator(device=device).manual_seed(0)
    value = torch.randn(B, S, H, D, device=device, generator=g).bfloat16().requires_grad_()
    ref = torch.rand(B, Lq, L, 4, device=device, generator=g).bfloat16()
    ref[..., 2:] = ref[..., 2:] * 0.3 + 0.02
    ref.requires_grad_()
    off = torch.randn(B, Lq, H, L, P, 2, device=device, generator=g).bfloat16().requires_grad_()
    logits = torch.randn(B, Lq, H, L * P, device=device, generator=g).bfloat16().requires_grad_()
    gout = torch.randn(B, Lq, H * D, device=device, generator=g).bfloat16()

    def ours():
        out = msda(value, shapes, ref, off, logits)
        out.backward(gout)

    def baseline():  # fp32 grid_sample path incl. the bf16 -> fp32 casts
        out = msda_reference(value, shapes, ref, off, logits)
        out.backward(gout.float())

    if quick:   # a few launches only (for profiler captures)
        for _ in range(3):
            ours()
        torch.cuda.synchronize()
        return []
    t_ours = time_ms(ours, warmup=3, iters=5)
    t_base = time_ms(baseline, warmup=2, iters=3, reps=3)
    row = {"op": "msda_fwd_bwd", "B": B, "S": S, "H": H, "D": D, "Lq": Lq, "levels": L, "points": P,
           "ms_ours": round(t_ours, 3), "ms_fp32_grid_sample": round(t_base, 3), "speedup": round(t_base / t_ours, 2)}
    mod = _reference_module()
    if mod is not None:
        # the reference's own K1 / K2 (ms_deform_attn_op.cpp: bf16 -> fp32 casts, im2col forward,
        # col2im backward) on the same sampling locations and softmaxed weights
        from .msda import _locations
        with torch.no_grad():
            loc = _locations(ref.float(), off.float()).bfloat16()
            attn = torch.softmax(logits.float().view(B, Lq, H, L * P), -1).view(B, Lq, H, L, P).bfloat16()
        spatial = torch.tensor(shapes, dtype=torch.int64, device=device)
        starts = torch.tensor([0] + [h * w for h, w in shapes[:-1]], dtype=torch.int64, device=device).cumsum(0)

        def reference():
            mod.msda_fwd_bwd(value.detach(), spatial, starts, loc, attn, gout, 64)
        row["ms_reference_k1k2"] = round(time_ms(reference, warmup=2, iters=5), 3)
        row["speedup_vs_reference"] = round(row["ms_reference_k1k2"] / t_ours, 2)
    return [row]


def _reference_module():
    """The reference build of bench.py's reference arm (baseline/_ref), or None when absent."""
    import glob
    import importlib.util
    import os
    root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    so = sorted(glob.glob(os.path.join(root, "baseline", "_ref", "mmltk_ref*.so")))
    if not so:
        return None
    spec = importlib.util.spec_from_file_location("mmltk_ref", so[0])
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


# (name, batch*windows or batch*groups, heads, length, head dim): RF-DETR-M batch 8
ATTN_SHAPES = [("dec.self_attn", 104, 8, 300, 32), ("vit.window", 32, 6, 325, 64), ("vit.global", 8, 6, 1300, 64),
               ("vit.window.b1", 4, 6, 325, 64), ("vit.global.b1", 1, 6, 1300, 64)]


def bench_attn(device="cuda", quick=False):
    """Forward + backward of the step's attention shapes under each SDPA backend.  ``quick``:
    three launches of the tcgen05 forward on the ViT global shape, untimed (profiler runs)."""
    if quick:
        g = torch.Generator(device=device).manual_seed(0)
        if quick == "short":
            # forward + backward of the short-sequence kernels on the decoder self-attention shape
            from .attention import short_attention
            N, H, L, D = 104, 8, 300, 32
            qkv = torch.randn(N * L, 3 * H * D, device=device, generator=g).bfloat16().requires_grad_()
            go = torch.randn(N * L, H * D, device=device, generator=g).bfloat16()
            for _ in range(3):
                torch.autograd.grad(short_attention(qkv, None, (0, H * D, 2 * H * D), N, L, H, D), (qkv,), go)
            torch.cuda.synchronize()
            return [{"op": "attention", "shape": "dec.self_attn", "quick": True}]
        from .attention import qkv_attention_tc
        qkv = torch.randn(8, 1300, 3 * 384, device=device, generator=g).bfloat16()
        with torch.no_grad():
            for _ in range(3):
                qkv_attention_tc(qkv, 6)
        torch.cuda.synchronize()
        return [{"op": "attention", "shape": "vit.global", "quick": True}]
    from torch.nn.attention import SDPBackend, sdpa_kernel
    import torch.nn.functional as F
    rows = []
    for name, N, H, L, D in ATTN_SHAPES:
        g = torch.Generator(device=device).manual_seed(0)
        q, k, v = (torch.randn(N, H, L, D, device=device, generator=g).bfloat16().requires_grad_() for _ in range(3))
        go = torch.randn(N, H, L, D, device=device, generator=g).bfloat16()
        row = {"op": "attention", "shape": name, "N": N, "H": H, "L": L, "D": D}
        for be in (SDPBackend.CUDNN_ATTENTION, SDPBackend.FLASH_ATTENTION, SDPBackend.EFFICIENT_ATTENTION):
            def fwd():
                with sdpa_kernel([be]):
                    return F.scaled_dot_product_attention(q, k, v)

            def both():
                fwd().backward(go)
            try:
                row[be.name.lower() + "_fwd_ms"] = round(time_ms(fwd, warmup=3, iters=10), 4)
                row[be.name.lower() + "_fwd_bwd_ms"] = round(time_ms(both, warmup=3, iters=10), 4)
            except RuntimeError as e:   # backend unavailable for this shape / arch
                row[be.name.lower()] = f"unavailable: {str(e).splitlines()[0][:80]}"
        if L <= 384 and D in (32, 64):
            # the packed projection layout [N * L, 3 * H * D], forward and forward + backward as CUDA-graph
            # replays: the framework's short-sequence tcgen05 kernels against cuDNN on strided views
            from .attention import _split, short_attention
            C = H * D
            qkv = torch.randn(N * L, 3 * C, device=device, generator=g).bfloat16().requires_grad_()
            gos = torch.randn(N * L, C, device=device, generator=g).bfloat16()

            def cudnn_pk():
                with sdpa_kernel([SDPBackend.CUDNN_ATTENTION]):
                    return F.scaled_dot_product_attention(*_split(qkv.view(N, L, 3 * C), H))

            def short_pk():
                return short_attention(qkv, None, (0, C, 2 * C), N, L, H, D)

            from ._ext import kernels
            for v in (1, 2):    # forward variants: whole score row per CTA / ping-pong warpgroups
                kernels().attn_short_set_fwd_variant(v)
                with torch.no_grad():
                    row[f"packed_short_v{v}_fwd_ms"] = round(time_graph_ms(short_pk), 4)
            kernels().attn_short_set_fwd_variant(2)
            for tag, f in (("cudnn", cudnn_pk), ("short", short_pk)):
                with torch.no_grad():
                    row[f"packed_{tag}_fwd_ms"] = round(time_graph_ms(f), 4)
                go_t = gos if tag == "short" else gos.view(N, L, H, D).transpose(1, 2)
                row[f"packed_{tag}_fwd_bwd_ms"] = round(time_graph_ms(
                    lambda: torch.autograd.grad(f(), (qkv,), go_t)), 4)
            if D == 32:
                # head-dim-32 backward kernels: one block at a time (1) / pipelined half-blocks (2)
                for v in (1, 2):
                    kernels().attn_short_set_bwd_variant(v)
                    row[f"packed_short_bwd_v{v}_fwd_bwd_ms"] = round(time_graph_ms(
                        lambda: torch.autograd.grad(short_pk(), (qkv,), gos)), 4)
                kernels().attn_short_set_bwd_variant(2)
        if D == 64:
            # forward on the packed projection layout: the tcgen05 kernel vs cuDNN on strided views
            from .attention import _split, qkv_attention_tc
            qkv = torch.randn(N, L, 3 * H * D, device=device, generator=g).bfloat16()
            with torch.no_grad():     # device time: CUDA-graph replays (the host is out of the loop)
                with sdpa_kernel([SDPBackend.CUDNN_ATTENTION]):
                    row["packed_cudnn_fwd_ms"] = round(time_graph_ms(
                        lambda: F.scaled_dot_product_attention(*_split(qkv, H))), 4)
                from ._ext import kernels
                for variant in (2, 1):     # two CTAs per SM (168 registers) / one CTA per SM
                    kernels().attn_tc_set_variant(variant)
                    row[f"packed_tc{variant}_fwd_ms"] = round(time_graph_ms(lambda: qkv_attention_tc(qkv, H)), 4)
                    row[f"tc{variant}_blocks_per_sm"] = kernels().attn_tc_blocks_per_sm()
                kernels().attn_tc_set_variant(2)
        rows.append(row)
    return rows


def _criterion_case(device, B=8, groups=13, Qg=300, C=91, layers=4, kmax=10):
    """Synthetic decoder outputs of RF-DETR-M training (main + aux layers + two-stage layer) and
    targets: the criterion's matcher cost, assignment solver and matched / dense losses."""
    from ..config import config_from_preset
    from ..criterion import SetCriterion
    from ..data.synthetic import synthetic_targets
    cfg = config_from_preset("rf-detr-medium")
    g = torch.Generator(device="cpu").manual_seed(0)
    Q = groups * Qg

    def layer():
        lg = (torch.randn(B, Q, C, generator=g) * 2).to(device, torch.bfloat16).requires_grad_()
        bx = torch.rand(B, Q, 4, generator=g).clamp(0.05, 0.95).to(device, torch.bfloat16).requires_grad_()
        return {"pred_logits": lg, "pred_boxes": bx}

    out = layer()
    out["aux_outputs"] = [layer() for _ in range(layers - 1)]
    out["enc_outputs"] = layer()
    targets = synthetic_targets(B, g, 1, kmax, C - 1, kmax).to(device)
    leaves = [l[k] for l in [out] + out["aux_outputs"] + [out["enc_outputs"]] for k in ("pred_logits", "pred_boxes")]
    return SetCriterion(cfg), out, targets, leaves


def bench_kernels(device="cuda", quick=False):
    """Small-footprint launches of the step's memory-bound kernels (one op at a time, a few hundred MB
    on the device): LayerNorm forward / backward on the ViT shape, the criterion (matcher cost + GPU
    assignment solver + fused matched losses, forward and backward) on RF-DETR-M's training outputs,
    and the top-k post-process.  ``quick``: three launches of each, untimed (profiler captures)."""
    from ._ext import kernels
    from .norm import layer_norm
    from ..infer.postprocess import postprocess
    g = torch.Generator(device=device).manual_seed(0)
    x = torch.randn(10400, 384, device=device, generator=g).bfloat16().requires_grad_()
    w = (1 + 0.1 * torch.randn(384, device=device, generator=g)).bfloat16().requires_grad_()
    b = (0.1 * torch.randn(384, device=device, generator=g)).bfloat16().requires_grad_()
    gy = torch.randn(10400, 384, device=device, generator=g).bfloat16()
    crit, out, targets, leaves = _criterion_case(device)
    logits = torch.randn(8, 300, 91, device=device, generator=g).bfloat16()
    boxes = torch.rand(8, 300, 4, device=device, generator=g).bfloat16()

    def ln():
        torch.autograd.grad(layer_norm(x, w, b, 1e-6), (x, w, b), gy)

    def crit_step():
        losses, _ = crit(out, targets, training=True)
        torch.autograd.grad(crit.weighted(losses), leaves)

    def post():
        postprocess({"pred_logits": logits, "pred_boxes": boxes}, 100, (560, 560), masks=False)

    # single-launch column reductions: the decoder FFN's ReLU backward with its bias gradient, and
    # the ViT MLP's bias gradient (column sum of the 1536-wide gradient)
    k = kernels()
    g_relu = torch.randn(31200, 2048, device=device, generator=g).bfloat16()
    pre_relu = torch.randn(31200, 2048, device=device, generator=g).bfloat16()
    g_mlp = torch.randn(10400, 1536, device=device, generator=g).bfloat16()

    def relu_bwd_bias():
        k.act_bwd_bias(g_relu, pre_relu, 2)

    def colsum():
        k.colsum(g_mlp, torch.float32)

    # the step's glue kernels on RF-DETR-M's batch-8 shapes: the four tapped ViT stages normalised
    # straight into the [B, 36, 36, 4 * 384] projector input, the decoder's per-group LayerNorm, the
    # two-stage gather's backward (index-add of 31200 rows into 10368), the grouped bias gradient,
    # the row top-k of the proposal scores, the patch unfold of a 576^2 batch and the projector's
    # LayerNorm + SiLU
    from .norm import concat_channels, grouped_layer_norm, taps_layer_norm
    from .linear import gather_rows
    states = [torch.randn(32, 325, 384, device=device, generator=g).bfloat16().requires_grad_() for _ in range(4)]
    g_taps = torch.randn(8, 36, 36, 4 * 384, device=device, generator=g).bfloat16()
    xg = torch.randn(13, 8, 300, 256, device=device, generator=g).bfloat16().requires_grad_()
    wg = (1 + 0.1 * torch.randn(13, 256, device=device, generator=g)).bfloat16().requires_grad_()
    bg = (0.1 * torch.randn(13, 256, device=device, generator=g)).bfloat16().requires_grad_()
    gyg = torch.randn_like(xg)
    table = torch.randn(10368, 256, device=device, generator=g).bfloat16().requires_grad_()
    rows_idx = torch.randint(0, 10368, (31200,), device=device, generator=g)
    g_rows = torch.randn(31200, 256, device=device, generator=g).bfloat16()
    g_grp = torch.randn(13, 2400, 256, device=device, generator=g).bfloat16()
    scores = torch.randn(13, 8, 1296, device=device, generator=g).bfloat16()
    img = torch.randn(8, 3, 576, 576, device=device, generator=g).bfloat16()
    xs = torch.randn(8 * 72 * 72, 256, device=device, generator=g).bfloat16().requires_grad_()
    ws = (1 + 0.1 * torch.randn(256, device=device, generator=g)).bfloat16().requires_grad_()
    bs = (0.1 * torch.randn(256, device=device, generator=g)).bfloat16().requires_grad_()
    gys = torch.randn_like(xs)

    def taps():
        feats = concat_channels(taps_layer_norm(states, w, b, 1e-6, 8, 2, 18, 18))
        torch.autograd.grad(feats, states + [w, b], g_taps)

    def grouped_ln():
        torch.autograd.grad(grouped_layer_norm(xg, wg, bg, 1e-5), (xg, wg, bg), gyg)

    def gather_bwd():
        torch.autograd.grad(gather_rows(table, rows_idx), (table,), g_rows)

    def colsum_grp():
        k.colsum_grouped(g_grp, torch.float32)

    def topk():
        k.row_topk(scores, 300)

    def unfold():
        k.patch_unfold(img, 16)

    def ln_silu():
        torch.autograd.grad(layer_norm(xs, ws, bs, 1e-6, act="silu"), (xs, ws, bs), gys)

    cases = [("layer_norm.fwd_bwd.vit-384", ln), ("criterion.fwd_bwd.rf-detr-m-b8", crit_step),
             ("postprocess.topk100.b8", post), ("colreduce.relu_bwd_bias.dec-ffn1-31200x2048", relu_bwd_bias),
             ("colreduce.colsum.vit-mlp-10400x1536", colsum),
             ("layer_norm.taps.fwd_bwd.4x32x325x384", taps),
             ("layer_norm.grouped.fwd_bwd.13x2400x256", grouped_ln),
             ("gather_rows.bwd.31200-of-10368x256", gather_bwd),
             ("colreduce.colsum_grouped.13x2400x256", colsum_grp),
             ("row_topk.k300.104x1296", topk),
             ("patch_unfold.p16.8x3x576x576", unfold),
             ("layer_norm.silu.fwd_bwd.41472x256", ln_silu)]
    rows = []
    for name, fn in cases:
        if quick:
            for _ in range(3):
                fn()
            torch.cuda.synchronize()
            rows.append({"op": name, "quick": True})
        else:
            rows.append({"op": name, "ms": round(time_ms(fn, warmup=3, iters=10), 4)})
    return rows


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("what", choices=["gemm", "msda", "attn", "kernels"])
    ap.add_argument("--shape", default=None, help="run one GEMM shape (see GEMM_SHAPES)")
    ap.add_argument("--quick", nargs="?", const="default", default=None,
                    help="launch a few times without timing (profiler runs); attn: '--quick short' runs the "
                         "short-sequence kernels on the decoder shape")
    ap.add_argument("--variant", type=int, default=0,
                    help="gemm: 0 tile variant per shape, 1 single-CTA tiles, 2 CTA-pair tiles")
    args = ap.parse_args()
    if args.what == "gemm":
        from ._ext import kernels
        kernels().gemm_tc_set_variant(args.variant)
        rows = bench_gemm(only=args.shape, quick=bool(args.quick))
    elif args.what == "msda":
        rows = bench_msda(quick=bool(args.quick))
    elif args.what == "kernels":
        rows = bench_kernels(quick=bool(args.quick))
    else:
        rows = bench_attn(quick=args.quick)
    for r in rows:
        print(json.dumps(r))


if __name__ == "__main__":
    main()
