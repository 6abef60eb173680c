"""Muon with an auxiliary AdamW (the reference's ``NativeMuonWithAuxAdam``).

Reference: `src/rfdetr/training/native_optimizer.cpp:30-39,271-290,424-445,709-812`,
eligibility `src/rfdetr/training/train.cpp:942-955`.  Hidden 2-D / 4-D weights
(not embeddings, tokens, query / refpoint tables, class / box heads or the
segmentation head) take Muon: momentum lerp, Nesterov blend, orthogonalisation
by five Newton-Schulz iterations with the quintic coefficients
(3.4445, -4.7750, 2.0315) published with Muon (K. Jordan et al., 2024) on the
bf16 matrix normalised by its Frobenius norm (+1e-7), the wide orientation, a
``sqrt(max(1, rows / cols))`` scale, decoupled weight decay.  Everything else
takes AdamW with betas (0.9, 0.95), eps 1e-10.

B200 design: parameters with the same matrix shape are stacked and
orthogonalised together with batched GEMMs (one chain per shape class instead
of one per parameter), which keeps the tensor cores busy on the many
384x384 / 1536x384 ViT matrices.  On the GPU the chain runs on the framework's
batched tcgen05 GEMM (``ops.gemm.bmm_nt`` / ``bmm_nn_mn``: every stacked matrix
through one pair of tensor maps, the quintic's coefficients in the alpha / beta
epilogue); shapes it does not take (a reduction that is not a multiple of 64)
use the library's batched GEMM.  State and updates are fp32 on the master
weights.  Eager only, like the reference.
"""
from __future__ import annotations

import math
from collections import defaultdict
from typing import Dict, List, Optional, Sequence, Tuple

import torch

__all__ = ["is_muon_hidden_weight", "newton_schulz5", "MuonAux", "NS_COEFFS"]

NS_COEFFS = (3.4445, -4.7750, 2.0315)
NS_STEPS = 5
NORM_EPS = 1e-7
AUX_BETAS = (0.9, 0.95)
AUX_EPS = 1e-10

_EXCLUDE = ("embeddings", "position_embeddings", "cls_token", "mask_token", "query_feat", "refpoint_embed",
            "class_embed", "bbox_embed", "segmentation_head")


def is_muon_hidden_weight(name: str, p: torch.Tensor) -> bool:
    if p.dim() not in (2, 4) or ".weight" not in name and not name.endswith("_weight"):
        return False
    return not any(e in name for e in _EXCLUDE)


def newton_schulz5(g: torch.Tensor, steps: int = NS_STEPS) -> torch.Tensor:
    """g [..., r, c] -> approximately the orthogonal polar factor, bf16 arithmetic."""
    a, b, c = NS_COEFFS
    x = g.to(torch.bfloat16)
    t = x.shape[-2] > x.shape[-1]
    if t:
        x = x.transpose(-2, -1)
    x = x / (x.flatten(-2).norm(dim=-1)[..., None, None] + NORM_EPS)
    lead = x.shape[:-2]
    x = x.reshape(-1, *x.shape[-2:]).contiguous()
    if x.is_cuda:
        # batched tcgen05 products (every matrix of the shape class in one launch), the polynomial's
        # scaling and sums in their alpha / beta epilogues; G = X X^T is symmetric, so G.G = G G^T
        from ..ops.gemm import bmm_nn_mn, bmm_nt
        for _ in range(steps):
            gram = bmm_nt(x, x)                                        # X X^T
            poly = bmm_nt(gram, gram, alpha=c, beta=b, res=gram)       # c*G.G + b*G
            x = bmm_nn_mn(poly, x, alpha=1.0, beta=a, res=x)           # P.X + a*X
        steps = 0
    for _ in range(steps):
        # three GEMMs per step, the polynomial's scaling and sums in their alpha / beta epilogues
        gram = torch.bmm(x, x.transpose(-2, -1))
        poly = torch.baddbmm(gram, gram, gram, beta=b, alpha=c)       # b*G + c*G.G
        x = torch.baddbmm(x, poly, x, beta=a, alpha=1.0)              # a*X + P.X
    x = x.reshape(*lead, *x.shape[-2:])
    if t:
        x = x.transpose(-2, -1)
    return x


class MuonAux:
    """Optimizer over a list of fp32 master tensors (updated in place)."""

    def __init__(self, names: Sequence[str], masters: Sequence[torch.Tensor], group_of: Sequence[int],
                 groups: Sequence[dict], momentum: float = 0.95, nesterov: bool = True):
        self.names = list(names)
        self.masters = list(masters)
        self.group_of = list(group_of)
        self.groups = [dict(g) for g in groups]
        self.momentum = momentum
        self.nesterov = nesterov
        self.use_muon = [is_muon_hidden_weight(n, p) for n, p in zip(self.names, self.masters)]
        self.state: List[Dict[str, torch.Tensor]] = []
        for m, mu in zip(self.masters, self.use_muon):
            if mu:
                self.state.append({"momentum_buffer": torch.zeros_like(m, dtype=torch.float32)})
            else:
                self.state.append({"exp_avg": torch.zeros_like(m, dtype=torch.float32),
                                   "exp_avg_sq": torch.zeros_like(m, dtype=torch.float32), "step": 0})
        # shape classes for the batched orthogonalisation; a fused q/k/v weight is three
        # matrices (the reference keeps separate query / key / value Linears)
        self.classes: Dict[Tuple[int, int], List[Tuple[int, int]]] = defaultdict(list)
        for i, (n, m, mu) in enumerate(zip(self.names, self.masters, self.use_muon)):
            if mu:
                blocks = 3 if n.endswith("qkv_weight") else 1
                r = m.shape[0] // blocks
                for k in range(blocks):
                    self.classes[(r, m.numel() // m.shape[0])].append((i, k))

    @torch.no_grad()
    def step(self, grads: Sequence[torch.Tensor], lr_scale: float = 1.0, momentum: Optional[float] = None) -> None:
        beta = self.momentum if momentum is None else momentum
        lrs = [g["lr"] * lr_scale for g in self.groups]
        for i, mu in enumerate(self.use_muon):   # momentum first (whole tensors)
            if mu:
                self.state[i]["momentum_buffer"].lerp_(grads[i].float().view_as(self.masters[i]), 1 - beta)
        for (r, c), blocks in self.classes.items():
            ups = []
            for i, k in blocks:
                g = grads[i].float().reshape(-1, c)[k * r:(k + 1) * r]
                mb = self.state[i]["momentum_buffer"].reshape(-1, c)[k * r:(k + 1) * r]
                ups.append(g.lerp(mb, beta) if self.nesterov else mb.clone())
            o = newton_schulz5(torch.stack(ups)).float() * math.sqrt(max(1.0, r / c))
            for j, (i, k) in enumerate(blocks):
                gi = self.group_of[i]
                lr, wd = lrs[gi], self.groups[gi]["weight_decay"]
                m = self.masters[i].view(-1, c)[k * r:(k + 1) * r]
                if wd:
                    m.mul_(1 - lr * wd)
                m.add_(o[j], alpha=-lr)
        b1, b2 = AUX_BETAS
        for i, mu in enumerate(self.use_muon):
            if mu:
                continue
            st = self.state[i]
            st["step"] += 1
            g = grads[i].float().view_as(self.masters[i])
            st["exp_avg"].lerp_(g, 1 - b1)
            st["exp_avg_sq"].lerp_(g * g, 1 - b2)
            c1 = 1 - b1 ** st["step"]
            c2 = 1 - b2 ** st["step"]
            upd = (st["exp_avg"] / c1) / ((st["exp_avg_sq"] / c2).sqrt() + AUX_EPS)
            gi = self.group_of[i]
            lr, wd = lrs[gi], self.groups[gi]["weight_decay"]
            if wd:
                self.masters[i].mul_(1 - lr * wd)
            self.masters[i].add_(upd, alpha=-lr)

    def state_dict(self) -> dict:
        d = {"kind": "muon", "entry_count": len(self.names)}
        for i, (n, st) in enumerate(zip(self.names, self.state)):
            e = {"name": n, "use_muon": bool(self.use_muon[i])}
            for k, v in st.items():
                e[k] = v.detach().cpu() if isinstance(v, torch.Tensor) else int(v)
            d[f"entry_{i:06d}"] = e
        return d

    def load_state_dict(self, d: dict) -> None:
        if d.get("kind") != "muon":
            raise ValueError(f"resume: optimizer kind {d.get('kind')!r} does not match 'muon'")
        by_name = {d[f"entry_{i:06d}"]["name"]: d[f"entry_{i:06d}"] for i in range(int(d["entry_count"]))}
        for n, st in zip(self.names, self.state):
            e = by_name.get(n)
            if e is None:
                raise ValueError(f"resume: optimizer state has no entry for {n}")
            for k in st:
                if isinstance(st[k], torch.Tensor):
                    st[k].copy_(e[k].view_as(st[k]))
                else:
                    st[k] = int(e[k])
