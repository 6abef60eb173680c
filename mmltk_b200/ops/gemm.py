"""bf16 GEMM entry points used by the dense layers (fp32 accumulation).

``gemm_nt(a [M,K], b [N,K], bias)`` -> a b^T (+ bias)   (forward)
``gemm_nn(a [M,N], b [N,K])``        -> a b               (input gradient)
``gemm_tn(a [M,N], b [M,K])``        -> a^T b             (weight gradient)

Shapes that fit the framework's sm_100a kernel (``gemm_tc``: TMA loads into
128B-swizzled shared memory, ``tcgen05.mma`` with the accumulator in tensor
memory, epilogue through ``tcgen05.ld``) run on it; everything else runs on
cuBLAS through torch.
"""
from __future__ import annotations

import os

import torch

from ._ext import kernels

__all__ = ["gemm_nt", "gemm_nn", "gemm_tn", "set_tc_gemm", "tc_gemm_enabled"]

_state = {"enabled": os.environ.get("MMLTK_TC_GEMM", "1") != "0", "checked": False, "have": False}


def set_tc_gemm(flag: bool) -> None:
    _state["enabled"] = bool(flag)


def tc_gemm_enabled() -> bool:
    if not _state["checked"]:
        _state["have"] = hasattr(kernels(), "gemm_tc")
        _state["checked"] = True
    return _state["enabled"] and _state["have"]


def _tc_fits(M, N, K):
    return M % 128 == 0 and N % 64 == 0 and K % 64 == 0


def gemm_nt(a: torch.Tensor, b: torch.Tensor, bias=None) -> torch.Tensor:
    M, K = a.shape
    N = b.shape[0]
    if tc_gemm_enabled() and _tc_fits(M, N, K):
        return kernels().gemm_tc(a, b, bias, False, False)
    if bias is None:
        return torch.mm(a, b.t())
    return torch.addmm(bias, a, b.t())


def gemm_nn(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    M, N = a.shape
    K = b.shape[1]
    if tc_gemm_enabled() and _tc_fits(M, K, N):
        return kernels().gemm_tc(a, b, None, False, True)
    return torch.mm(a, b)


def gemm_tn(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    M, N = a.shape
    K = b.shape[1]
    if tc_gemm_enabled() and _tc_fits(N, K, M):
        return kernels().gemm_tc(a, b, None, True, True)
    return torch.mm(a.t(), b)
