"""Two-stage deformable transformer with Group-DETR queries.

Reference: `NativeTransformerImpl` / `NativeDecoderImpl` / `NativeDecoderLayerImpl`
/ `MSDeformAttnImpl` / `gen_encoder_output_proposals`
(`src/rfdetr/layers/model.cpp:808-1363`).

Numerics kept from the reference:
* decoder layer: self-attn (nn.MultiheadAttention layout, 8 heads) on
  ``q = k = tgt + query_pos, v = tgt``; in training the 13 Group-DETR groups are
  attended independently; post-LN; MSDeformAttn; FFN (ReLU); post-LN;
* lite refpoint refine: the reference points and the ``ref_point_head`` query
  position are computed once from the initial refpoints;
* two-stage proposals ``(x+0.5)/W, wh = 0.05 * 2**lvl``, validity (0.01, 0.99);
  per-group ``enc_output`` Linear -> LN -> class Linear / bbox MLP with bbox
  reparameterisation, top-k by max class logit.

B200 design: the 13 per-group encoder heads are stacked parameters evaluated
as batched GEMMs (one launch per head stage instead of 13); their checkpoint
keys are still ``enc_output.<g>.weight`` etc. through state-dict hooks.  The
proposal grid is computed once per feature shape and cached on the device.
"""
from __future__ import annotations

import math
from typing import List, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from .. import ops
from ..ops import kernels
from ..config import RfDetrConfig


class Mlp(nn.Module):
    """`RfDetrMlpImpl` (reference `src/rfdetr/layers/modules.cpp:61-83`): Linear+ReLU stack."""

    def __init__(self, din: int, dh: int, dout: int, n: int):
        super().__init__()
        dims = [din] + [dh] * (n - 1)
        outs = [dh] * (n - 1) + [dout]
        self.layers = nn.ModuleList(nn.Linear(a, b) for a, b in zip(dims, outs))

    def forward(self, x):
        n = len(self.layers)
        for i, l in enumerate(self.layers):
            if i + 1 < n:
                x = ops.linear(x, l.weight, l.bias, act="relu")
            else:
                x = ops.linear(x, l.weight, l.bias)
        return x


def gen_sineembed_for_position(pos: torch.Tensor, dim: int = 128) -> torch.Tensor:
    """Sine embedding of (x, y[, w, h]) -> [..., 2*dim or 4*dim] (reference `model.cpp:234-261`):
    blocks y, x[, w, h], entries sin / cos of v * 2 pi / 10000^(2i/dim).  One fused kernel each
    way on CUDA (bf16 out); the fp32 torch expression on CPU."""
    return ops.sine_embed(pos, dim)


class _ReparamBoxesFn(torch.autograd.Function):
    """reparam_boxes with its backward written out: two concatenated gradients instead of autograd's
    zero-filled full-size buffer per slice of ``delta`` / ``base`` and the sums of their pieces."""

    @staticmethod
    def forward(ctx, delta, base):
        dxy, dwh = delta[..., :2], delta[..., 2:]
        bxy, bwh = base[..., :2], base[..., 2:]
        e = dwh.exp()
        ctx.save_for_backward(dxy, bwh, e)
        return torch.cat([dxy * bwh + bxy, e * bwh], -1)

    @staticmethod
    def backward(ctx, g):
        dxy, bwh, e = ctx.saved_tensors
        gxy, gwh = g[..., :2], g[..., 2:]
        gwh_e = gwh * e
        gd = torch.cat([gxy * bwh, gwh_e * bwh], -1) if ctx.needs_input_grad[0] else None
        gb = torch.cat([gxy, gxy * dxy + gwh_e], -1) if ctx.needs_input_grad[1] else None
        return gd, gb


def reparam_boxes(delta: torch.Tensor, base: torch.Tensor) -> torch.Tensor:
    """bbox reparameterisation: cxcy = d_xy * base_wh + base_xy, wh = exp(d_wh) * base_wh."""
    if torch.is_grad_enabled() and (delta.requires_grad or base.requires_grad):
        return _ReparamBoxesFn.apply(delta, base)
    cxcy = delta[..., :2] * base[..., 2:] + base[..., :2]
    wh = delta[..., 2:].exp() * base[..., 2:]
    return torch.cat([cxcy, wh], -1)


class MSDeformAttn(nn.Module):
    def __init__(self, d_model: int, n_levels: int, n_heads: int, n_points: int):
        super().__init__()
        self.d_model, self.n_levels, self.n_heads, self.n_points = d_model, n_levels, n_heads, n_points
        self.sampling_offsets = nn.Linear(d_model, n_heads * n_levels * n_points * 2)
        self.attention_weights = nn.Linear(d_model, n_heads * n_levels * n_points)
        self.value_proj = nn.Linear(d_model, d_model)
        self.output_proj = nn.Linear(d_model, d_model)
        self.reset_parameters()

    def reset_parameters(self):
        """Grid init (reference `model.cpp:873-895`)."""
        with torch.no_grad():
            self.sampling_offsets.weight.zero_()
            thetas = torch.arange(self.n_heads, dtype=torch.float32) * (2.0 * math.pi / self.n_heads)
            grid = torch.stack([thetas.cos(), thetas.sin()], -1)
            grid = (grid / grid.abs().max(-1, keepdim=True)[0]).view(self.n_heads, 1, 1, 2)
            grid = grid.repeat(1, self.n_levels, self.n_points, 1)
            for i in range(self.n_points):
                grid[:, :, i, :] *= i + 1
            self.sampling_offsets.bias.copy_(grid.view(-1))
            self.attention_weights.weight.zero_()
            self.attention_weights.bias.zero_()
            nn.init.xavier_uniform_(self.value_proj.weight)
            self.value_proj.bias.zero_()
            nn.init.xavier_uniform_(self.output_proj.weight)
            self.output_proj.bias.zero_()

    def forward(self, query, ref, value_in, shapes, padding_mask=None, defer_bias: bool = False):
        """``defer_bias``: return (output without the output projection's bias, that bias) for a
        consumer that adds it itself (the decoder's fused residual + norm)."""
        B, Lq, _ = query.shape
        S = value_in.shape[1]
        H, L, P = self.n_heads, self.n_levels, self.n_points
        value = ops.linear(value_in, self.value_proj.weight, self.value_proj.bias)
        if padding_mask is not None:
            value = value.masked_fill(padding_mask[..., None], 0.0)
        value = value.view(B, S, H, self.d_model // H)
        off, logits = ops.linear_pair(query, self.sampling_offsets.weight, self.sampling_offsets.bias,
                                      self.attention_weights.weight, self.attention_weights.bias)
        off, logits = off.view(B, Lq, H, L, P, 2), logits.view(B, Lq, H, L * P)
        out = ops.msda(value, shapes, ref, off, logits)
        if defer_bias:
            return ops.linear(out.to(query.dtype), self.output_proj.weight, None), self.output_proj.bias
        return ops.linear(out.to(query.dtype), self.output_proj.weight, self.output_proj.bias)


class DecoderLayer(nn.Module):
    def __init__(self, cfg: RfDetrConfig):
        super().__init__()
        d = cfg.hidden_dim
        self.group_detr = max(1, cfg.group_detr)
        self.self_attn = nn.MultiheadAttention(d, cfg.sa_nheads, dropout=0.0)
        self.norm1 = nn.LayerNorm(d)
        self.cross_attn = MSDeformAttn(d, cfg.num_feature_levels, cfg.ca_nheads, cfg.dec_n_points)
        self.linear1 = nn.Linear(d, cfg.dim_feedforward)
        self.linear2 = nn.Linear(cfg.dim_feedforward, d)
        self.norm2 = nn.LayerNorm(d)
        self.norm3 = nn.LayerNorm(d)

    def _self_attention(self, tgt, query_pos, groups, tgt_pos=None):
        B, Q, d = tgt.shape
        H = self.self_attn.num_heads
        Dh = d // H
        w, b = self.self_attn.in_proj_weight, self.self_attn.in_proj_bias
        # split (not slices): the weight / bias gradients are one concatenation each instead of
        # zero-filled full-size buffers per slice, copies and an accumulation
        w_qk, w_v = w.split([2 * d, d])
        b_qk, b_v = b.split([2 * d, d])
        qk = ops.linear(tgt_pos if tgt_pos is not None else tgt + query_pos, w_qk, b_qk)  # [B, Q, 2d]
        v = ops.linear(tgt, w_v, b_v)                           # [B, Q, d]
        Qg = Q // groups
        qk2, v2 = qk.view(B * Q, 2 * d), v.view(B * Q, d)
        if ops.short_attention_ok(Qg, Dh, qk2, v2):
            # rows b*Q + g*Qg + i = sequence b*G + g: attention never crosses a group; q / k / v are
            # read straight out of the projections and the gradients land in them
            o = ops.short_attention(qk2, v2, (0, d, 0), B * groups, Qg, H, Dh).view(B, Q, d)
            return ops.linear(o, self.self_attn.out_proj.weight, None), self.self_attn.out_proj.bias
        # [B, G, Qg, H, Dh] -> [B*G, H, Qg, Dh]: attention never crosses a group; on cuDNN with
        # the backward writing straight into the two projections' gradients
        o = ops.qk_split_attention(qk, v, B * groups, Qg, H)
        if o is not None:
            return ops.linear(o, self.self_attn.out_proj.weight, None), self.self_attn.out_proj.bias
        # split (not two slices): its backward is one concatenation instead of two
        # zero-filled full-width buffers, two copies and an add
        qh, kh = qk.split(d, dim=-1)
        q = qh.reshape(B * groups, Qg, H, Dh).transpose(1, 2)
        k = kh.reshape(B * groups, Qg, H, Dh).transpose(1, 2)
        vv = v.reshape(B * groups, Qg, H, Dh).transpose(1, 2)
        o = ops.attention(q, k, vv).transpose(1, 2).reshape(B, Q, d)
        # the output projection's bias is added (and its gradient reduced) by the following norm
        return ops.linear(o, self.self_attn.out_proj.weight, None), self.self_attn.out_proj.bias

    def forward(self, tgt, query_pos, ref, memory, shapes, padding_mask, groups, tgt_pos=None, want_pos=False):
        """Post-norm layer.  ``tgt_pos`` = tgt + query_pos when the caller has it already;
        ``want_pos`` also returns out + query_pos (the next layer's self-attention input), made by
        the last norm's kernel.  Residual adds are fused into the norms."""
        # each branch's last linear runs without its bias; the fused add + norm adds it and reduces
        # its gradient in the norm's backward kernel
        sa, sa_b = self._self_attention(tgt, query_pos, groups, tgt_pos)
        x, x_pos = ops.add_layer_norm(tgt, sa, self.norm1.weight, self.norm1.bias, 1e-5, pos=query_pos, rbias=sa_b)
        ca, ca_b = self.cross_attn(x_pos, ref, memory, shapes, padding_mask, defer_bias=True)
        x = ops.add_layer_norm(x, ca, self.norm2.weight, self.norm2.bias, 1e-5, rbias=ca_b)
        # FFN + residual + post-norm as one node (its backward needs no add of the two x gradients)
        return ops.ffn_add_norm(x, self.linear1.weight, self.linear1.bias, self.linear2.weight, self.linear2.bias,
                                self.norm3.weight, self.norm3.bias, 1e-5, pos=query_pos if want_pos else None)


class Decoder(nn.Module):
    def __init__(self, cfg: RfDetrConfig):
        super().__init__()
        self.cfg = cfg
        self.layers = nn.ModuleList(DecoderLayer(cfg) for _ in range(max(1, cfg.dec_layers)))
        self.norm = nn.LayerNorm(cfg.hidden_dim)
        self.ref_point_head = Mlp(2 * cfg.hidden_dim, cfg.hidden_dim, cfg.hidden_dim, 2)

    def forward(self, tgt, memory, refpoints, shapes, padding_mask, valid_ratios, groups, bbox_embed=None):
        cfg = self.cfg
        L = len(shapes)

        def reference(r):
            vr = valid_ratios if valid_ratios is not None else torch.ones(r.shape[0], L, 2, device=r.device,
                                                                           dtype=r.dtype)
            rin = r[:, :, None, :4] * torch.cat([vr, vr], -1)[:, None].to(r.dtype)  # [B,Q,L,4]
            sine = gen_sineembed_for_position(rin[:, :, 0], cfg.hidden_dim // 2).to(tgt.dtype)
            return rin, self.ref_point_head(sine)

        out = tgt
        refs = refpoints
        intermediate = []
        hs_refs = [refpoints]
        if cfg.lite_refpoint_refine:
            rin, qpos = reference(refs if cfg.bbox_reparam else refs.sigmoid())
        out_pos = None   # out + qpos, from the previous layer's last norm
        for li, layer in enumerate(self.layers):
            if not cfg.lite_refpoint_refine:
                rin, qpos = reference(refs if cfg.bbox_reparam else refs.sigmoid())
                out_pos = None
            # the next layer reuses this layer's qpos only under lite refinement
            chain = cfg.lite_refpoint_refine and li + 1 < len(self.layers)
            res = layer(out, qpos, rin, memory, shapes, padding_mask, groups, tgt_pos=out_pos, want_pos=chain)
            out, out_pos = res if chain else (res, None)
            if not cfg.lite_refpoint_refine and bbox_embed is not None:
                delta = bbox_embed(out)
                new = reparam_boxes(delta, refs) if cfg.bbox_reparam else refs + delta
                if li != len(self.layers) - 1:
                    hs_refs.append(new)
                refs = new.detach()
            intermediate.append(ops.layer_norm(out, self.norm.weight, self.norm.bias, 1e-5))
        if bbox_embed is not None and not cfg.lite_refpoint_refine:
            return torch.stack(intermediate), torch.stack(hs_refs)
        return torch.stack(intermediate), refs.unsqueeze(0)


class GroupedLinear(nn.Module):
    """G independent Linear layers stored as one [G, out, in] parameter.

    State dict keys are ``<g>.weight`` / ``<g>.bias`` (a ModuleList of Linear in
    the reference checkpoint)."""

    def __init__(self, groups: int, din: int, dout: int):
        super().__init__()
        self.groups = groups
        ref = [nn.Linear(din, dout) for _ in range(groups)]
        self.weight = nn.Parameter(torch.stack([l.weight.data for l in ref]))
        self.bias = nn.Parameter(torch.stack([l.bias.data for l in ref]))

        def save_hook(mod, state, prefix, md):
            w = state.pop(prefix + "weight")
            b = state.pop(prefix + "bias")
            for g in range(w.shape[0]):
                state[f"{prefix}{g}.weight"] = w[g]
                state[f"{prefix}{g}.bias"] = b[g]

        def load_hook(state, prefix, md, strict, missing, unexpected, errors):
            ks = [f"{prefix}{g}.weight" for g in range(self.groups)]
            if all(k in state for k in ks):
                state[prefix + "weight"] = torch.stack([state.pop(k) for k in ks])
                state[prefix + "bias"] = torch.stack([state.pop(f"{prefix}{g}.bias") for g in range(self.groups)])

        self._register_state_dict_hook(save_hook)
        self._register_load_state_dict_pre_hook(load_hook)

    def forward(self, x: torch.Tensor, groups: int, act=None) -> torch.Tensor:
        """x: [G', B, N, din] (one slice per group) or [B, N, din] (shared) -> [groups, B, N, dout]."""
        if groups == self.weight.shape[0]:   # no slice: a full-range slice's backward still zero-fills + copies
            return grouped_linear(x, self.weight, self.bias, act)
        return grouped_linear(x, self.weight[:groups], self.bias[:groups], act)


class _GroupedLinearFn(torch.autograd.Function):
    """y[g] = x[g] w[g]^T + b[g] for stacked x [G, R, din], w [G, dout, din], b [G, dout].
    Forward and input gradient run as batched products on the tcgen05 kernel (``bmm_nt`` /
    ``bmm_nn_mn``, library GEMM where the kernel does not take the shape); the weight gradient
    reduces over the R rows of every group (not a multiple of 64 in general) on the library's
    batched GEMM."""

    @staticmethod
    def forward(ctx, x, w, b):
        from ..ops.gemm import bmm_nt
        ctx.save_for_backward(x, w)
        return bmm_nt(x, w, b)

    @staticmethod
    def backward(ctx, gy):
        from ..ops.gemm import bmm_nn_mn
        x, w = ctx.saved_tensors
        gy = gy.contiguous()
        dx = bmm_nn_mn(gy, w) if ctx.needs_input_grad[0] else None
        dw = torch.bmm(gy.transpose(1, 2), x) if ctx.needs_input_grad[1] else None
        db = None
        if ctx.needs_input_grad[2]:
            # per-group bias gradients in one column-reduction launch (fp32 accumulation)
            k = kernels()
            db = (k.colsum_grouped(gy) if gy.is_cuda and gy.shape[2] % 8 == 0 and hasattr(k, "colsum_grouped")
                  else gy.sum(1))
        return dx, dw, db


def grouped_linear(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor, act=None) -> torch.Tensor:
    """Per-group affine maps: x [G, B, N, din] or [B, N, din] (shared), w [G, dout, din], b [G, dout]."""
    w = w.to(x.dtype)
    b = b.to(x.dtype)
    dout = w.shape[1]
    pad = (-dout) % 8 if x.is_cuda else 0
    if pad:   # odd widths (91 classes, 4 box deltas) would put cuBLAS on its unaligned kernels
        w = F.pad(w, (0, 0, 0, pad))
        b = F.pad(b, (0, pad))
    G = w.shape[0]
    shared = x.dim() == 3
    if shared:
        B, N, C = x.shape
        x = x.unsqueeze(0).expand(G, B, N, C)
    _, B, N, C = x.shape
    if x.is_cuda and x.dtype == torch.bfloat16 and not shared:
        # batched tcgen05 products: forward and input gradient on the framework's kernel
        y = _GroupedLinearFn.apply(x.reshape(G, B * N, C).contiguous(), w.contiguous(), b.contiguous())
        y = y.view(G, B, N, -1)
    else:
        # batched GEMM with the bias folded in (beta = 1 on a broadcast bias)
        y = torch.baddbmm(b[:, None, :], x.reshape(G, B * N, C), w.transpose(1, 2)).view(G, B, N, -1)
    if pad:
        y = y[..., :dout]
    if act == "relu":
        y = F.relu(y)
    return y


class GroupedLayerNorm(nn.Module):
    def __init__(self, groups: int, dim: int):
        super().__init__()
        self.groups = groups
        self.weight = nn.Parameter(torch.ones(groups, dim))
        self.bias = nn.Parameter(torch.zeros(groups, dim))

        def save_hook(mod, state, prefix, md):
            w = state.pop(prefix + "weight")
            b = state.pop(prefix + "bias")
            for g in range(w.shape[0]):
                state[f"{prefix}{g}.weight"] = w[g]
                state[f"{prefix}{g}.bias"] = b[g]

        def load_hook(state, prefix, md, strict, missing, unexpected, errors):
            ks = [f"{prefix}{g}.weight" for g in range(self.groups)]
            if all(k in state for k in ks):
                state[prefix + "weight"] = torch.stack([state.pop(k) for k in ks])
                state[prefix + "bias"] = torch.stack([state.pop(f"{prefix}{g}.bias") for g in range(self.groups)])

        self._register_state_dict_hook(save_hook)
        self._register_load_state_dict_pre_hook(load_hook)

    def forward(self, x, groups):
        # x [G, B, N, C]: normalise with group g's affine (one kernel each way on the GPU)
        if groups == self.groups:     # the parameters themselves (their gradients go straight to .grad)
            return ops.grouped_layer_norm(x, self.weight, self.bias, 1e-5)
        return ops.grouped_layer_norm(x, self.weight[:groups], self.bias[:groups], 1e-5)


class GroupedMlp(nn.Module):
    """G independent 3-layer box MLPs; keys ``<g>.layers.<i>.weight``."""

    def __init__(self, groups: int, din: int, dh: int, dout: int, n: int):
        super().__init__()
        self.groups = groups
        dims = [din] + [dh] * (n - 1)
        outs = [dh] * (n - 1) + [dout]
        self.layers = nn.ModuleList(GroupedLinear(groups, a, b) for a, b in zip(dims, outs))
        # re-key: GroupedLinear hooks emit `layers.<i>.<g>.weight`; the checkpoint wants `<g>.layers.<i>.weight`

        def save_hook(mod, state, prefix, md):
            n_l = len(self.layers)
            for i in range(n_l):
                for g in range(self.groups):
                    for t in ("weight", "bias"):
                        k = f"{prefix}layers.{i}.{g}.{t}"
                        if k in state:
                            state[f"{prefix}{g}.layers.{i}.{t}"] = state.pop(k)

        def load_hook(state, prefix, md, strict, missing, unexpected, errors):
            for i in range(len(self.layers)):
                for g in range(self.groups):
                    for t in ("weight", "bias"):
                        k = f"{prefix}{g}.layers.{i}.{t}"
                        if k in state:
                            state[f"{prefix}layers.{i}.{g}.{t}"] = state.pop(k)

        self._register_state_dict_hook(save_hook)
        self._register_load_state_dict_pre_hook(load_hook)

    def forward(self, x, groups):
        n = len(self.layers)
        for i, l in enumerate(self.layers):
            x = l(x, groups, act="relu" if i + 1 < n else None)
        return x


_proposal_cache = {}


def encoder_proposals(shapes, batch: int, device, dtype, unsigmoid: bool):
    """Full-valid two-stage proposals (reference `model.cpp:1076-1139`), cached per shape.

    Returns (proposals [1, S, 4], valid [1, S, 1])."""
    key = (tuple(shapes), str(device), dtype, unsigmoid)
    hit = _proposal_cache.get(key)
    if hit is not None:
        return hit
    props = []
    for lvl, (h, w) in enumerate(shapes):
        gy, gx = torch.meshgrid(torch.arange(h, dtype=torch.float32, device=device),
                                torch.arange(w, dtype=torch.float32, device=device), indexing="ij")
        grid = torch.stack([(gx + 0.5) / w, (gy + 0.5) / h], -1)
        wh = torch.full_like(grid, 0.05 * (2.0 ** lvl))
        props.append(torch.cat([grid, wh], -1).view(1, -1, 4))
    p = torch.cat(props, 1)
    valid = ((p > 0.01) & (p < 0.99)).all(-1, keepdim=True)
    if unsigmoid:
        p = torch.log(p / (1 - p)).masked_fill(~valid, float("inf"))
    else:
        p = p.masked_fill(~valid, 0.0)
    out = (p.to(dtype), valid)
    _proposal_cache[key] = out
    return out


class Transformer(nn.Module):
    def __init__(self, cfg: RfDetrConfig):
        super().__init__()
        self.cfg = cfg
        G = max(1, cfg.group_detr)
        d = cfg.hidden_dim
        self.decoder = Decoder(cfg)
        self.enc_output = GroupedLinear(G, d, d)
        self.enc_output_norm = GroupedLayerNorm(G, d)
        self.enc_out_class_embed = GroupedLinear(G, d, max(1, cfg.num_classes))
        self.enc_out_bbox_embed = GroupedMlp(G, d, d, 4, 3)
        prior = -math.log((1 - 0.01) / 0.01)
        with torch.no_grad():
            self.enc_out_class_embed.bias.fill_(prior)

    def forward(self, feats: List[torch.Tensor], refpoint_embed, query_feat, training: bool, bbox_embed=None):
        """feats: channels-last [B, h, w, C] per level.  Returns dict with hs [Ldec,B,Q,C], refs, enc_* ."""
        cfg = self.cfg
        B = feats[0].shape[0]
        shapes = [(f.shape[1], f.shape[2]) for f in feats]
        flat = [f.reshape(B, -1, f.shape[-1]) for f in feats]
        memory = flat[0] if len(flat) == 1 else torch.cat(flat, 1)                 # [B, S, C]
        groups = max(1, cfg.group_detr) if training else 1
        out = {"shapes": shapes}
        refpoints = refpoint_embed.unsqueeze(0).expand(B, -1, -1)
        if cfg.two_stage:
            props, valid = encoder_proposals(shapes, B, memory.device, memory.dtype, not cfg.bbox_reparam)
            out_mem = memory.masked_fill(~valid, 0.0)
            # Selection pass over every token, without autograd: only the top-k indices leave it.
            with torch.no_grad():
                topk = self._select(out_mem, groups)                                   # [G, B, k]
                k = topk.shape[2]
            # Differentiable pass on the selected tokens only: the head is per token, so recomputing
            # enc_output + norm + box MLP on the k chosen rows gives the same values (and gradients)
            # as gathering them from the full pass, at k / S of the cost.
            S, C = out_mem.shape[1], out_mem.shape[2]
            # rows of the flattened [B*S, C] memory (its backward is one index_add into a [B*S, C]
            # gradient, not a scatter into a group-expanded [G, B, S, C] buffer summed over groups)
            rows = (torch.arange(B, device=topk.device, dtype=topk.dtype)[None, :, None] * S + topk).reshape(-1)
            mem_in = ops.gather_rows(out_mem.reshape(B * S, C), rows).view(groups, B, k, C)   # [G, B, k, C]
            mem_sel = self.enc_output_norm(self.enc_output(mem_in, groups), groups)    # [G, B, k, C]
            delta = self.enc_out_bbox_embed(mem_sel, groups)                            # [G, B, k, 4]
            props_sel = props.expand(B, -1, -1).unsqueeze(0).expand(groups, -1, -1, -1).gather(
                2, topk[..., None].expand(-1, -1, -1, 4))                               # [G, B, k, 4]
            if cfg.bbox_reparam:
                boxes = reparam_boxes(delta, props_sel)
            else:
                boxes = delta + props_sel
            # group-major query order [B, G*k, .]
            enc_boxes = boxes.permute(1, 0, 2, 3).reshape(B, groups * k, 4)
            enc_mem = mem_sel.permute(1, 0, 2, 3).reshape(B, groups * k, -1)
            out["enc_boxes"] = enc_boxes if cfg.bbox_reparam else enc_boxes.sigmoid()
            out["enc_memory"] = enc_mem
            ts = enc_boxes.detach()
            n_ts = ts.shape[1]
            head = refpoints[:, :n_ts]
            if cfg.bbox_reparam:
                head = reparam_boxes(head.to(ts.dtype), ts)
            else:
                head = head + ts
            refpoints = torch.cat([head, refpoints[:, n_ts:].to(head.dtype)], 1)
        tgt = query_feat.unsqueeze(0).expand(B, -1, -1).to(memory.dtype)
        hs, refs = self.decoder(tgt, memory, refpoints.to(memory.dtype), shapes, None, None, groups, bbox_embed)
        out["hs"] = hs
        out["refs"] = refs
        out["memory"] = memory
        return out

    def _select(self, out_mem: torch.Tensor, groups: int) -> torch.Tensor:
        """Top-k token indices per group by the best class logit of the two-stage head.

        * every group's ``enc_output`` in ONE GEMM over the shared memory tokens:
          [B*S, C] x [C, G*C] (no per-group copy of the input);
        * LayerNorm without affine over each C-wide slice; the norm's per-group affine is
          folded into the class head: W' = W diag(gamma), b' = W beta + b;
        * class logits as a strided batched GEMM over the groups; the class dimension is
          padded to a multiple of 8 with zero weights and -inf bias, so the max over the
          padded, contiguous rows equals the max over the real classes; on the GPU the GEMM's
          epilogue reduces each row to its maximum (the logits are never stored).
        """
        B, S, C = out_mem.shape
        G = groups
        dt = out_mem.dtype
        w_all = self.enc_output.weight[:G].to(dt).reshape(G * C, C)
        b_all = self.enc_output.bias[:G].to(dt).reshape(G * C)
        h = ops.linear(out_mem, w_all, b_all)                                  # [B, S, G*C]
        unit = h.new_ones(C)
        hn = ops.layer_norm(h.view(B, S, G, C), unit, torch.zeros_like(unit), 1e-5)
        del h
        wc = self.enc_out_class_embed.weight[:G].float()
        gam = self.enc_output_norm.weight[:G].float()
        bet = self.enc_output_norm.bias[:G].float()
        w_f = wc * gam[:, None, :]
        b_f = self.enc_out_class_embed.bias[:G].float() + torch.einsum("gkc,gc->gk", wc, bet)
        K = w_f.shape[1]
        pad = (-K) % 8
        if pad:
            w_f = F.pad(w_f, (0, 0, 0, pad))
            b_f = F.pad(b_f, (0, pad), value=float("-inf"))
        if hn.is_cuda:
            # one batched tcgen05 GEMM over the groups (group g's operand is columns [g*C, g*C + C) of
            # the shared rows) whose epilogue keeps only each row's best logit: the [G, B*S, K] logits
            # are never written.  Rounded to the compute dtype, like a max over rounded logits.
            from ..ops.gemm import bmm_nt_rowmax
            best = bmm_nt_rowmax(hn.view(B * S, G * C), w_f.to(dt).contiguous(), b_f.to(dt).contiguous(), C,
                                 B * S).to(dt).view(G, B, S)
        else:
            x = hn.view(B * S, G, C).transpose(0, 1)                           # [G, B*S, C], row stride G*C
            cls = torch.baddbmm(b_f.to(dt)[:, None, :], x, w_f.to(dt).transpose(1, 2))   # [G, B*S, K+pad]
            best = cls.amax(-1).view(G, B, S)
        k = min(self.cfg.num_queries, S)
        # (the framework's row_topk kernel gives the same indices but measured 35 us against the
        # library's 2 x 13.5 us for 104 rows of 1296: its per-row sort is barrier-bound at one CTA
        # per row)
        return best.topk(k, dim=2)[1]

    def encoder_class_logits(self, enc_memory: torch.Tensor, groups: int) -> torch.Tensor:
        B, Q, C = enc_memory.shape
        x = enc_memory.view(B, groups, Q // groups, C).permute(1, 0, 2, 3)   # [G, B, k, C]
        logits = self.enc_out_class_embed(x, groups)                         # [G, B, k, K]
        return logits.permute(1, 0, 2, 3).reshape(B, Q, -1)
