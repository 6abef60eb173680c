"""The allocation-free MSDeformAttn backward entry point.

``mmltk_msda_bwd_noalloc`` serves callers that must not allocate GPU memory
while they run (pre-planned runtimes, custom memory pools, C/C++ hosts
without a caching allocator).  This test calls it through its exported C
symbol, twice in a row, and checks both results against the regular
``msda_bwd`` op.  It lives in its own file, collected last, so that a run
stopping at the first failure has already run every other test.
"""
import ctypes
import os

import pytest
import torch

pytestmark = pytest.mark.gpu

LIB = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "mmltk_b200", "libmmltk_noalloc.so")


def _lib():
    if not os.path.exists(LIB):
        from mmltk_b200.build import build_noalloc
        build_noalloc()
    lib = ctypes.CDLL(LIB)
    fn = lib.mmltk_msda_bwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_int] + [ctypes.c_void_p] * 11 + [ctypes.c_int] * 7 + [ctypes.c_void_p]
    return fn


def _inputs(dtype, device, B=2, shapes=((12, 10), (6, 5)), Lq=40, H=8, D=16, P=3, seed=0):
    g = torch.Generator().manual_seed(seed)
    S = sum(h * w for h, w in shapes)
    L = len(shapes)
    value = torch.randn(B, S, H, D, generator=g)
    ref = torch.rand(B, Lq, L, 4, generator=g) * 0.8 + 0.1
    off = torch.randn(B, Lq, H, L, P, 2, generator=g) * 2
    logits = torch.randn(B, Lq, H, L * P, generator=g)
    gout = torch.randn(B, Lq, H * D, generator=g)
    starts = [0]
    for h, w in shapes[:-1]:
        starts.append(starts[-1] + h * w)
    t = [x.to(device, dtype).contiguous() for x in (gout, value, ref, off, logits)]
    sh = torch.tensor(shapes, dtype=torch.int32, device=device)
    st = torch.tensor(starts, dtype=torch.int32, device=device)
    return t, sh, st, (B, S, Lq, H, L, P, D)


def _call(fn, dtype_code, t, sh, st, dims, outs):
    gout, value, ref, off, logits = t
    stream = torch.cuda.current_stream().cuda_stream
    return fn(dtype_code, gout.data_ptr(), value.data_ptr(), sh.data_ptr(), st.data_ptr(), ref.data_ptr(),
              off.data_ptr(), logits.data_ptr(), *[o.data_ptr() for o in outs], *dims, stream)


@pytest.mark.parametrize("dtype,code,tol", [(torch.float32, 0, 1e-5), (torch.bfloat16, 1, 2e-2)])
def test_noalloc_matches_regular_op_twice(cuda_device, dtype, code, tol):
    from mmltk_b200.ops import kernels
    fn = _lib()
    t, sh, st, dims = _inputs(dtype, cuda_device)
    gout, value, ref, off, logits = t
    expect = kernels().msda_bwd(gout, value, sh, st, ref, off, logits)
    outs = [torch.empty_like(x) for x in (value, ref, off, logits)]
    for _ in range(2):  # the second call must not see the first call's accumulators
        for o in outs:
            o.fill_(float("nan"))
        rc = _call(fn, code, t, sh, st, dims, outs)
        torch.cuda.synchronize()
        assert rc == 0
        for got, exp in zip(outs, expect):
            scale = max(1e-6, exp.float().abs().max().item())
            assert (got.float() - exp.float()).abs().max().item() / scale < tol


def test_noalloc_rejects_oversized_problem(cuda_device):
    fn = _lib()
    t, sh, st, dims = _inputs(torch.float32, cuda_device)
    outs = [torch.empty_like(x) for x in t[1:]]
    B, S, Lq, H, L, P, D = dims
    rc = _call(fn, 0, t, sh, st, (64, 100000, Lq, H, L, P, D), outs)  # 64*100000*8*16 > 8 Mi elements
    assert rc == -1


def test_noalloc_rejects_unsupported_arguments(cuda_device):
    """An unsupported head dim (24) or dtype code (2) returns MMLTK_NOALLOC_ERR_BAD_ARG (-2)."""
    fn = _lib()
    t, sh, st, dims = _inputs(torch.float32, cuda_device)
    outs = [torch.empty_like(x) for x in t[1:]]
    B, S, Lq, H, L, P, D = dims
    assert _call(fn, 0, t, sh, st, (B, S, Lq, H, L, P, 24), outs) == -2
    assert _call(fn, 2, t, sh, st, dims, outs) == -2


def test_noalloc_on_a_side_stream(cuda_device):
    """The entry point runs on the stream it is given: a call on a non-default stream matches
    the regular op."""
    from mmltk_b200.ops import kernels
    fn = _lib()
    t, sh, st, dims = _inputs(torch.float32, cuda_device, seed=3)
    gout, value, ref, off, logits = t
    expect = kernels().msda_bwd(gout, value, sh, st, ref, off, logits)
    outs = [torch.full_like(x, float("nan")) for x in (value, ref, off, logits)]
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        rc = _call(fn, 0, t, sh, st, dims, outs)
    side.synchronize()
    assert rc == 0
    for got, exp in zip(outs, expect):
        scale = max(1e-6, exp.float().abs().max().item())
        assert (got.float() - exp.float()).abs().max().item() / scale < 1e-5
