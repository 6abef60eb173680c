"""RGBA overlay kernels (csrc/kernels/overlay.cu) vs their CPU restatements (mmltk_b200.infer.overlay)."""
import pytest
import torch

from mmltk_b200.infer import overlay as ovl

pytestmark = pytest.mark.gpu


def _pair(h=97, w=131, fill=0):
    base = torch.full((h, w, 4), fill, dtype=torch.uint8)
    return base.clone(), base.clone().cuda()


def _mismatch(cpu, gpu):
    """fraction of pixels whose RGBA differs by more than 1"""
    d = (cpu.int() - gpu.cpu().int()).abs().amax(-1)
    return (d > 1).float().mean().item()


def test_overlay_detections(cuda_device):
    torch.manual_seed(0)
    a, b = _pair()
    boxes = torch.tensor([[10.0, 12.0, 60.0, 50.0], [40.0, 30.0, 120.0, 90.0], [-5.0, 70.0, 20.0, 200.0]])
    colors = torch.tensor([[255, 0, 0], [0, 255, 0], [0, 0, 255]], dtype=torch.uint8)
    masks = (torch.rand(3, 97, 131) > 0.7).to(torch.uint8)
    ovl.overlay_detections(a, boxes, colors, masks, 2, 100)
    ovl.overlay_detections(b, boxes.cuda(), colors.cuda(), masks.cuda(), 2, 100)
    assert _mismatch(a, b) == 0.0
    assert (a[..., 3] == 255).any() and (a[..., 3] == 100).any()


@pytest.mark.parametrize("channels,swap", [(3, False), (4, False), (4, True)])
def test_composite_rgba(cuda_device, channels, swap):
    torch.manual_seed(1)
    dst = torch.randint(0, 256, (64, 80, channels), dtype=torch.uint8)
    src = torch.randint(0, 256, (64, 80, 4), dtype=torch.uint8)
    g = dst.cuda()
    ovl.composite_rgba(dst, src, swap)
    ovl.composite_rgba(g, src.cuda(), swap)
    assert (dst.int() - g.cpu().int()).abs().max().item() <= 1


def test_copy_rgb_to_rgba(cuda_device):
    src = torch.randint(0, 256, (33, 47, 3), dtype=torch.uint8)
    for swap in (False, True):
        assert torch.equal(ovl.copy_rgb_to_rgba(src, swap, 200), ovl.copy_rgb_to_rgba(src.cuda(), swap, 200).cpu())


def test_manual_mask_and_runs(cuda_device):
    torch.manual_seed(2)
    a, b = _pair()
    m = (torch.rand(40, 50) > 0.5).to(torch.uint8)
    ovl.manual_mask(a, 100, 70, m, (10, 20, 30, 200))          # partly off the right / bottom edge
    ovl.manual_mask(b, 100, 70, m.cuda(), (10, 20, 30, 200))
    assert torch.equal(a, b.cpu())
    runs = torch.tensor([[0, 7], [55, 30], [300, 120], [990, 50]], dtype=torch.int32)
    ovl.manual_mask_runs(a, -3, 5, 40, 25, runs, (1, 2, 3))
    ovl.manual_mask_runs(b, -3, 5, 40, 25, runs.cuda(), (1, 2, 3))
    assert torch.equal(a, b.cpu())


@pytest.mark.parametrize("t", [1, 3])
def test_box_outline_and_handles(cuda_device, t):
    a, b = _pair()
    for box in ([10, 20, 70, 60], [-20, -10, 200, 50], [100, 80, 300, 300]):
        ovl.box_outline(a, box, t, (255, 255, 0))
        ovl.box_outline(b, box, t, (255, 255, 0))
    ovl.selection_handles(a, [30, 30, 90, 80], 2, (0, 255, 255, 180))
    ovl.selection_handles(b, [30, 30, 90, 80], 2, (0, 255, 255, 180))
    assert torch.equal(a, b.cpu())


@pytest.mark.parametrize("closed,t", [(False, 1), (True, 4)])
def test_polyline(cuda_device, closed, t):
    a, b = _pair()
    pts = torch.tensor([[5, 5], [120, 20], [60, 90], [10, 60], [-50, 300]], dtype=torch.int32)
    ovl.polyline(a, pts, closed, t, (200, 10, 10))
    ovl.polyline(b, pts.cuda(), closed, t, (200, 10, 10))
    assert _mismatch(a, b) < 0.002        # boundary pixels may round differently
    assert (a[..., 3] > 0).sum() > 100


def test_points_and_skeleton(cuda_device):
    a, b = _pair()
    pts = torch.tensor([[20, 20], [60, 30], [90, 80], [130, 96], [0, 0]], dtype=torch.int32)
    edges = torch.tensor([[0, 1], [1, 2], [2, 3], [3, 9]], dtype=torch.int32)   # the last edge is invalid: skipped
    ovl.points(a, pts, 4, (0, 0, 255))
    ovl.points(b, pts.cuda(), 4, (0, 0, 255))
    assert torch.equal(a, b.cpu())
    ovl.skeleton(a, pts, edges, 2, 3, (255, 128, 0))
    ovl.skeleton(b, pts.cuda(), edges.cuda(), 2, 3, (255, 128, 0))
    assert _mismatch(a, b) < 0.002


def test_label_colors(cuda_device):
    labels = torch.arange(-1, 200, dtype=torch.int32)
    cpu = ovl.label_colors(labels)
    gpu = ovl.label_colors(labels.cuda()).cpu()
    assert (cpu.int() - gpu.int()).abs().max().item() <= 1
    assert len({tuple(c) for c in cpu[1:12].tolist()}) == 11      # neighbouring ids get distinct colours
