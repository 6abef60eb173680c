"""Live path (lease ring, synthetic source, analyzer) and the image kernels
(letterbox, draw, vflip, composite, mask resize / pack / sample) against torch."""
import pytest
import torch

from mmltk_b200.infer import Predictor
from mmltk_b200.infer.visualize import draw_reference, letterbox, letterbox_reference, palette
from mmltk_b200.live import FrameAnalyzer, SyntheticFrameSource, run_live
from mmltk_b200.models.rfdetr import build_model
from mmltk_b200.ops import native


def test_lease_ring_latest_semantics():
    r = native().LeaseRing(3)
    a = r.acquire_write()
    r.publish(a, 1)
    b = r.acquire_write()
    r.publish(b, 2)
    c = r.acquire_write()
    r.publish(c, 3)
    d = r.acquire_write()            # every slot published: the oldest (seq 1) is recycled
    assert d == a and r.dropped() == 1
    r.publish(d, 4)
    slot, seq = r.acquire_latest(0.1)
    assert seq == 4 and r.dropped() == 3        # seqs 2 and 3 skipped
    with pytest.raises(Exception):
        r.publish(slot, 5)                      # leased, not writable
    r.release(slot)
    r.close()
    assert r.acquire_latest(0.05) is None


def test_live_cpu_end_to_end(tmp_path):
    torch.manual_seed(0)
    p = Predictor(build_model("rf-detr-tiny-test", num_classes=4), device="cpu")
    an = FrameAnalyzer(p, ["a", "b", "c", "d"], threshold=0.0)
    src = SyntheticFrameSource(96, 64, frames=6, seed=1)
    st = run_live(src, an, out_dir=str(tmp_path), save_every=2)
    assert st.frames_in == 6 and 1 <= st.frames_analyzed <= 6
    assert st.frames_analyzed + st.dropped >= 6 - 1
    assert any(p.suffix == ".png" for p in tmp_path.iterdir()) or st.frames_analyzed < 2


def test_draw_reference_outline_and_mask():
    img = torch.zeros(20, 30, 3, dtype=torch.uint8)
    boxes = torch.tensor([[5.0, 4.0, 15.0, 12.0]])
    col = torch.tensor([[200, 10, 10]], dtype=torch.uint8)
    m = torch.zeros(1, 20, 30, dtype=torch.uint8)
    m[0, 6:10, 7:12] = 1
    out = draw_reference(img, boxes, col, m, thickness=1, mask_alpha=0.5)
    assert out[4, 5].tolist() == [200, 10, 10]             # outline
    assert out[8, 9].tolist() == [100, 5, 5]                # mask blend
    assert out[0, 0].tolist() == [0, 0, 0]
    assert palette(torch.tensor([1, 2])).shape == (2, 3)


@pytest.mark.gpu
def test_letterbox_kernel_matches_reference():
    f = (torch.rand(37, 53, 3) * 255).to(torch.uint8)
    for (h, w) in [(64, 64), (48, 80)]:
        ref = letterbox_reference(f, h, w, bgr=True)
        out = letterbox(f.cuda(), h, w, bgr=True, normalize_bf16=False).cpu()
        assert (out - ref).abs().max() < 1e-4
        norm = letterbox(f.cuda(), h, w, bgr=True, normalize_bf16=True).float().cpu()
        mean = torch.tensor([0.485, 0.456, 0.406]).view(3, 1, 1)
        std = torch.tensor([0.229, 0.224, 0.225]).view(3, 1, 1)
        assert (norm - (ref - mean) / std).abs().max() < 0.03


@pytest.mark.gpu
def test_draw_and_image_kernels():
    from mmltk_b200.ops import kernels
    k = kernels()
    img = (torch.rand(40, 60, 3) * 255).to(torch.uint8)
    boxes = torch.tensor([[5.0, 10.0, 30.0, 35.0], [20.0, 2.0, 50.0, 20.0]])
    col = torch.tensor([[200, 10, 10], [10, 200, 10]], dtype=torch.uint8)
    m = torch.zeros(2, 40, 60, dtype=torch.uint8)
    m[0, 12:30, 8:25] = 1
    dev = img.cuda()
    k.draw_(dev, boxes, col, m, None, 2, 0.45, 2)
    ref = draw_reference(img, boxes, col, m, 2, 0.45)
    assert (dev.cpu().int() - ref.int()).abs().max() <= 1
    # label text pixels appear in the bar above box 0 when text is given
    dev2 = img.cuda()
    txt = torch.tensor([list(b"CAR 97%") + [0] * 5, list(b"B") + [0] * 11], dtype=torch.int8)
    k.draw_(dev2, boxes, col, None, txt, 2, 0.45, 1)
    assert not torch.equal(dev2.cpu(), draw_reference(img, boxes, col, None, 2, 0.45))
    # vflip matches a flip of the rows
    f = img.cuda()
    k.vflip_(f)
    assert torch.equal(f.cpu(), img.flip(0))
    # composite with alpha 0 / 255
    rgba = torch.zeros(40, 60, 4, dtype=torch.uint8, device="cuda")
    rgba[..., :3] = 255
    rgba[:20, :, 3] = 255
    c = img.cuda()
    k.composite_(c, rgba, False)
    assert torch.equal(c[:20].cpu(), torch.full((20, 60, 3), 255, dtype=torch.uint8))
    assert torch.equal(c[20:].cpu(), img[20:])
    # masks: resize / pack / sample
    mm = (torch.rand(3, 17, 23) > 0.5).to(torch.uint8)
    rs = k.resize_masks(mm.cuda(), 34, 46).cpu()
    assert torch.equal(rs[:, ::2, ::2], mm)
    bits = k.pack_masks(mm.cuda())
    assert bits.shape == (3, (17 * 23 + 63) // 64)
    pts = torch.rand(3, 50, 2)
    s = k.sample_packed_masks(bits, 17, 23, pts.cuda()).cpu()
    x = (pts[..., 0] * 23 - 0.5).round().long().clamp(0, 22)
    y = (pts[..., 1] * 17 - 0.5).round().long().clamp(0, 16)
    exp = torch.stack([mm[i, y[i], x[i]] for i in range(3)]).float()
    assert torch.equal(s, exp)


@pytest.mark.gpu
def test_live_gpu_graph_path(tmp_path):
    torch.manual_seed(0)
    p = Predictor(build_model("rf-detr-tiny-test", num_classes=4), device="cuda")
    an = FrameAnalyzer(p, ["a", "b", "c", "d"], threshold=0.0)
    st = run_live(SyntheticFrameSource(96, 64, frames=12, seed=2), an, out_dir=str(tmp_path), save_every=3)
    assert st.frames_analyzed >= 1 and st.latency_ms_p50 > 0
    p.release()


def test_overlay_cpu_raster_rules():
    """The CPU overlay rules the GPU kernels are tested against: a 1-pixel polyline is 8-connected
    along its length, handles are 8 squares, a disc of radius r covers the lattice points within r."""
    from mmltk_b200.infer import overlay as ovl
    ov = torch.zeros(40, 40, 4, dtype=torch.uint8)
    ovl.polyline(ov, torch.tensor([[2, 3], [35, 20]]), False, 1, (255, 0, 0))
    cols = ov[..., 3].nonzero()[:, 1].unique()
    assert cols.min().item() == 2 and cols.max().item() == 35 and len(cols) == 34
    ov.zero_()
    ovl.selection_handles(ov, [5, 5, 30, 30], 1, (0, 255, 0))
    assert int((ov[..., 3] > 0).sum()) == 8 * 9
    ov.zero_()
    ovl.points(ov, torch.tensor([[20, 20]]), 3, (0, 0, 255))
    assert int((ov[..., 3] > 0).sum()) == sum(1 for x in range(-3, 4) for y in range(-3, 4) if x * x + y * y <= 9)
