"""bf16 GEMM entry points used by the dense layers (fp32 accumulation).

``gemm_nt(a [M,K], b [N,K], bias)`` -> a b^T (+ bias)   (forward)
``gemm_nn(a [M,N], b [N,K])``        -> a b               (input gradient)
``gemm_tn(a [M,N], b [M,K])``        -> a^T b             (weight gradient)
``gemm_nt_epilogue(...)``            forward with a fused GELU / ReLU / LayerScale+residual epilogue

Shapes that fit the framework's sm_100a kernel (``gemm_tc``: TMA loads into
128B-swizzled shared memory, ``tcgen05.mma`` with the accumulator in tensor
memory, epilogue through ``tcgen05.ld``; K-major and MN-major operands, so no
transposes are materialised) run on it; anything else runs on cuBLAS.
"""
from __future__ import annotations

import os

import torch

from ._ext import kernels

__all__ = ["gemm_nt", "gemm_nn", "gemm_tn", "gemm_nt_epilogue", "set_tc_gemm", "tc_gemm_enabled",
           "bmm_nt", "bmm_nn_mn", "bmm_nt_rowmax"]

# The fused-epilogue forward products always run on the tcgen05 kernel (that is
# where fusing saves whole passes over memory); plain products (backward dgrad /
# wgrad) use cuBLAS unless MMLTK_TC_GEMM_ALL=1.
_state = {"enabled": os.environ.get("MMLTK_TC_GEMM", "1") != "0", "checked": False, "have": False,
          "all": os.environ.get("MMLTK_TC_GEMM_ALL", "0") == "1"}

EPI = {"gelu": 1, "relu": 2, "scale_residual": 3}


def set_tc_gemm(flag: bool, plain_products: bool = None) -> None:
    _state["enabled"] = bool(flag)
    if plain_products is not None:
        _state["all"] = bool(plain_products)


def tc_gemm_enabled() -> bool:
    if not _state["checked"]:
        _state["have"] = hasattr(kernels(), "gemm_tc")
        _state["checked"] = True
    return _state["enabled"] and _state["have"]


def _rowmajor(t):
    return t.stride(-1) == 1 and t.stride(0) % 8 == 0 and t.data_ptr() % 16 == 0


def _fits_nt(a, b):
    return tc_gemm_enabled() and a.shape[1] % 8 == 0 and b.shape[0] % 16 == 0 and _rowmajor(a) and _rowmajor(b)


def gemm_nt(a: torch.Tensor, b: torch.Tensor, bias=None) -> torch.Tensor:
    if _state["all"] and _fits_nt(a, b):
        return kernels().gemm_tc(a, b, bias, False, False)[0]
    if bias is None:
        return torch.mm(a, b.t())
    return torch.addmm(bias, a, b.t())


_SMS = {}


def num_sms() -> int:
    """Multiprocessors of the current device (cached per device)."""
    d = torch.cuda.current_device()
    if d not in _SMS:
        _SMS[d] = torch.cuda.get_device_properties(d).multi_processor_count
    return _SMS[d]


def _fills_gpu(M: int, N: int) -> bool:
    """True when a 128 x 128 tiling of the output gives at least half a wave of CTAs: below that
    (batch-1 inference shapes) the persistent one-tile-per-CTA GEMM leaves most SMs idle, and the
    library GEMM plus one elementwise pass is faster."""
    tiles = ((M + 127) // 128) * ((N + 127) // 128)
    return tiles * 2 >= num_sms()


def gemm_nt_epilogue(a, b, bias, epi: str, res=None, gamma=None, want_pre: bool = True, force: bool = False):
    """(out, pre) with out = act(a b^T + bias) or res + gamma * (a b^T + bias); pre = a b^T + bias
    (None unless ``want_pre``).  Returns None when the shape does not fit the tensor-core kernel
    (or, unless ``force``, is too small to fill the GPU with it); the caller then runs the library
    GEMM."""
    if not _fits_nt(a, b) or not (force or _fills_gpu(a.shape[0], b.shape[0])):
        return None
    r = kernels().gemm_tc(a, b, bias, False, False, EPI[epi], want_pre, res, gamma)
    return r[0], (r[1] if want_pre else None)


def gemm_nn(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    if (_state["all"] and tc_gemm_enabled() and a.shape[1] % 8 == 0 and b.shape[1] % 128 == 0 and _rowmajor(a)
            and _rowmajor(b)):
        return kernels().gemm_tc(a, b, None, False, True)[0]
    return torch.mm(a, b)


def gemm_tn(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    if (_state["all"] and tc_gemm_enabled() and a.shape[1] % 128 == 0 and b.shape[1] % 128 == 0 and _rowmajor(a)
            and _rowmajor(b)):
        return kernels().gemm_tc(a, b, None, True, True)[0]
    return torch.mm(a.t(), b)


def gemm_tn_acc(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """out += a^T b in one GEMM (beta = 1): weight gradients accumulated straight into .grad."""
    if (_state["all"] and tc_gemm_enabled() and a.shape[1] % 128 == 0 and b.shape[1] % 128 == 0 and _rowmajor(a)
            and _rowmajor(b) and out.is_contiguous() and out.data_ptr() % 16 == 0):
        kernels().gemm_tc_acc(a, b, True, True, out)
        return out
    return out.addmm_(a.t(), b)


# ---------------------------------------------------------------------------------------------
# Batched products on the tcgen05 kernel: every batch reads the same 2-D tensor maps at shifted
# tile coordinates, so stacked operands need no copies.  K must be a multiple of 64 (a K tail
# would read the next batch's operand); other shapes run on the library's batched GEMM.

def _bf16_rows(t):
    return t.is_cuda and t.dtype == torch.bfloat16 and t.stride(-1) == 1 and _rowmajor(t)


def bmm_nt(x: torch.Tensor, w: torch.Tensor, bias=None, alpha: float = 1.0, beta: float = 0.0, res=None):
    """x [G, M, K] @ w[G, N, K]^T (+ bias [G, N]); with ``res``: alpha * (x w^T + bias) + beta * res."""
    G, M, K = x.shape
    N = w.shape[1]
    if (tc_gemm_enabled() and K % 64 == 0 and N % 16 == 0 and x.is_contiguous() and w.is_contiguous()
            and _bf16_rows(x.view(G * M, K)) and _bf16_rows(w.view(G * N, K))):
        return kernels().gemm_tc_batched(x.view(G * M, K), w.view(G * N, K), bias, False, False, G, M, N, K,
                                         0, M, 0, N, 6 if res is not None else 0, alpha, beta, res)[0]
    y = torch.bmm(x, w.transpose(1, 2))
    if bias is not None:
        y = y + bias[:, None, :]
    return y if res is None else alpha * y + beta * res


def bmm_nn_mn(x: torch.Tensor, y: torch.Tensor, alpha: float = 1.0, beta: float = 0.0, res=None):
    """x [G, M, K] @ y [G, K, N] (y read MN-major, no transpose); with ``res``: alpha * x y + beta * res."""
    G, M, K = x.shape
    N = y.shape[2]
    if (tc_gemm_enabled() and K % 64 == 0 and N % 128 == 0 and x.is_contiguous() and y.is_contiguous()
            and _bf16_rows(x.view(G * M, K)) and _bf16_rows(y.view(G * K, N))):
        return kernels().gemm_tc_batched(x.view(G * M, K), y.view(G * K, N), None, False, True, G, M, N, K,
                                         0, M, K, 0, 6 if res is not None else 0, alpha, beta, res)[0]
    z = torch.bmm(x, y)
    return z if res is None else alpha * z + beta * res


def bmm_nt_rowmax(a: torch.Tensor, w: torch.Tensor, bias: torch.Tensor, col_shift: int, rows: int):
    """max over n of (A_g w_g^T + bias_g)[m, n] for every group g, without storing the products.

    ``a`` [rows, G * col_shift]: group g's [rows, K] operand starts at column g * col_shift
    (K = w.shape[2]); w [G, N, K], bias [G, N] (padding columns carry -inf bias).  Returns fp32
    [G, rows].  Falls back to the library GEMM + max when the kernel does not take the shape."""
    G, N, K = w.shape
    if (tc_gemm_enabled() and K % 64 == 0 and N % 16 == 0 and N <= 256 and w.is_contiguous()
            and _bf16_rows(a) and _bf16_rows(w.view(G * N, K))):
        r = kernels().gemm_tc_batched(a, w.view(G * N, K), bias, False, False, G, rows, N, K,
                                      col_shift, 0, 0, N, 7)[0]
        return torch.maximum(r[0], r[1])
    x = a.view(rows, G, col_shift)[..., :K].transpose(0, 1)
    return torch.baddbmm(bias[:, None, :], x, w.transpose(1, 2)).amax(-1).float()
