"""tcgen05 short-sequence attention (attn_short.cu) forward and backward vs the fp32 math
definition with autograd: the decoder layout (q / k in one projection, v in another, head dim 32)
and the packed ViT layout (q / k / v side by side, head dim 64), including partial 128-row tiles,
a single short tile and the 384-token maximum."""
import math

import pytest
import torch

from mmltk_b200.ops import kernels
from mmltk_b200.ops.attention import short_attention

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True, params=[2, 1], ids=["fwd-pingpong", "fwd-row"])
def fwd_variant(request):
    """Every test runs with both forward kernels: the ping-pong warpgroups over 128-key chunks
    (default) and the whole-score-row kernel."""
    k = kernels()
    old = k.attn_short_fwd_variant()
    k.attn_short_set_fwd_variant(request.param)
    yield request.param
    k.attn_short_set_fwd_variant(old)


def _oracle(q, k, v, go):
    """q/k/v/go fp32 [N, H, L, D] leaves -> (o, lse, dq, dk, dv)."""
    q, k, v = (t.detach().clone().requires_grad_() for t in (q, k, v))
    s = q @ k.transpose(-1, -2) / math.sqrt(q.shape[-1])
    lse = torch.logsumexp(s, -1)
    o = torch.softmax(s, -1) @ v
    o.backward(go)
    return o.detach(), lse.detach(), q.grad, k.grad, v.grad


def _close(got, ref, tol):
    err = (got.float() - ref.float()).abs().max().item()
    scale = max(1e-6, ref.float().abs().max().item())
    assert err / scale < tol, (err, scale)


def _heads(m, col, N, L, H, D):
    """[N*L, cols] matrix, head h at columns col + h*D -> [N, H, L, D] fp32."""
    return m[:, col:col + H * D].float().view(N, L, H, D).transpose(1, 2)


@pytest.fixture(params=[2, 1], ids=["bwd-pipelined", "bwd-blockwise"])
def bwd_variant(request):
    """Head-dim-32 tests run both backward kernels: pipelined half-blocks (default) and one block at
    a time."""
    k = kernels()
    old = k.attn_short_bwd_variant()
    k.attn_short_set_bwd_variant(request.param)
    yield request.param
    k.attn_short_set_bwd_variant(old)


@pytest.mark.parametrize("N,L,H", [(6, 300, 8), (3, 100, 8), (2, 129, 4), (2, 384, 8), (1, 17, 2), (2, 200, 3)])
def test_short_attention_split_d32(cuda_device, bwd_variant, N, L, H):
    torch.manual_seed(0)
    D = 32
    qk = (torch.randn(N * L, 2 * H * D, device=cuda_device) * 1.5).bfloat16().requires_grad_()
    v = torch.randn(N * L, H * D, device=cuda_device).bfloat16().requires_grad_()
    o = short_attention(qk, v, (0, H * D, 0), N, L, H, D)
    go = torch.randn_like(o)
    o.backward(go)
    assert kernels().attn_tc_status(torch.cuda.current_device()) == 0
    q_, k_, v_ = _heads(qk, 0, N, L, H, D), _heads(qk, H * D, N, L, H, D), _heads(v, 0, N, L, H, D)
    ro, _, dq, dk, dv = _oracle(q_, k_, v_, _heads(go, 0, N, L, H, D))
    _close(o.view(N, L, H, D).transpose(1, 2), ro, 2e-2)
    _close(_heads(qk.grad, 0, N, L, H, D), dq, 3e-2)
    _close(_heads(qk.grad, H * D, N, L, H, D), dk, 3e-2)
    _close(_heads(v.grad, 0, N, L, H, D), dv, 3e-2)


@pytest.mark.parametrize("N,L,H", [(3, 325, 6), (2, 128, 2), (2, 129, 3), (1, 384, 2), (4, 77, 6)])
def test_short_attention_packed_d64(cuda_device, N, L, H):
    torch.manual_seed(1)
    D = 64
    C = H * D
    qkv = (torch.randn(N * L, 3 * C, device=cuda_device) * 1.5).bfloat16().requires_grad_()
    o = short_attention(qkv, None, (0, C, 2 * C), N, L, H, D)
    go = torch.randn_like(o)
    o.backward(go)
    assert kernels().attn_tc_status(torch.cuda.current_device()) == 0
    q_, k_, v_ = (_heads(qkv, c, N, L, H, D) for c in (0, C, 2 * C))
    ro, _, dq, dk, dv = _oracle(q_, k_, v_, _heads(go, 0, N, L, H, D))
    _close(o.view(N, L, H, D).transpose(1, 2), ro, 2e-2)
    for c, ref in zip((0, C, 2 * C), (dq, dk, dv)):
        _close(_heads(qkv.grad, c, N, L, H, D), ref, 3e-2)


@pytest.mark.parametrize("D", [32, 64])
def test_short_attention_lse(cuda_device, D):
    torch.manual_seed(2)
    N, L, H = 3, 300, 4
    qkv = (torch.randn(N * L, 3 * H * D, device=cuda_device) * 2).bfloat16()
    o, lse = kernels().attn_short_fwd(qkv, 0, qkv, H * D, qkv, 2 * H * D, N, L, H, D)
    q_, k_, v_ = (_heads(qkv, c, N, L, H, D) for c in (0, H * D, 2 * H * D))
    _, rlse, *_ = _oracle(q_, k_, v_, torch.zeros(N, H, L, D, device=cuda_device))
    assert torch.allclose(lse, rlse, atol=2e-2, rtol=1e-3), (lse - rlse).abs().max().item()


def test_qkv_attention_takes_the_short_kernel_for_windows(cuda_device):
    """The ViT's packed attention routes windows (<= 384 tokens) to the short kernel, forward and
    backward, and still matches the math definition."""
    from mmltk_b200.ops.attention import qkv_attention, qkv_attention_reference
    torch.manual_seed(3)
    N, L, H = 4, 325, 6
    import importlib
    attn_mod = importlib.import_module("mmltk_b200.ops.attention")   # (the package re-exports a function of that name)
    qkv = (torch.randn(N, L, 3 * H * 64, device=cuda_device)).bfloat16().requires_grad_()
    old = attn_mod._SHORT_MODE
    attn_mod._SHORT_MODE = "1"
    try:
        o = qkv_attention(qkv, H)
    finally:
        attn_mod._SHORT_MODE = old
    fns = [type(o.grad_fn).__name__] + [type(f[0]).__name__ for f in o.grad_fn.next_functions if f[0] is not None]
    assert any("ShortAttn" in n for n in fns), fns
    ref = qkv_attention_reference(qkv.detach().float(), H)
    _close(o, ref, 2e-2)


@pytest.mark.parametrize("D", [32, 64])
def test_short_attention_running_max_moves(cuda_device, D):
    """Keys of the last 128-key chunk score far above the first chunk's, so the online softmax of the
    ping-pong kernel must move its running maximum and rescale the partial output in tensor memory."""
    torch.manual_seed(4)
    N, L, H = 2, 300, 2
    C = H * D
    qkv = torch.randn(N * L, 3 * C, device=cuda_device)
    kv = qkv.view(N, L, 3 * C)
    kv[:, 256:, C:2 * C] *= 6.0        # k rows of the third chunk
    qkv = qkv.bfloat16().requires_grad_()
    o = short_attention(qkv, None, (0, C, 2 * C), N, L, H, D)
    go = torch.randn_like(o)
    o.backward(go)
    assert kernels().attn_tc_status(torch.cuda.current_device()) == 0
    q_, k_, v_ = (_heads(qkv, c, N, L, H, D) for c in (0, C, 2 * C))
    ro, _, dq, dk, dv = _oracle(q_, k_, v_, _heads(go, 0, N, L, H, D))
    _close(o.view(N, L, H, D).transpose(1, 2), ro, 2e-2)
    for c, ref in zip((0, C, 2 * C), (dq, dk, dv)):
        _close(_heads(qkv.grad, c, N, L, H, D), ref, 4e-2)
