"""Data path: PNG codec, dataset compile -> reader -> loader round trip
(the reference's `tests/core/roundtrip.test.cpp` scenario), target packing."""
import json
import os

import pytest
import torch

from mmltk_b200.data.compiler import CompileError, compile_split, load_categories
from mmltk_b200.data.loader import BatchLoader, CompiledDataset
from mmltk_b200.data.source import write_synthetic_source
from mmltk_b200.ops import native


def test_png_roundtrip():
    img = (torch.rand(37, 53, 3) * 255).to(torch.uint8)
    data = native().encode_png(img)
    back = native().decode_png(data)
    assert torch.equal(back, img)


def test_png_matches_pil(tmp_path):
    from PIL import Image
    img = (torch.rand(21, 30, 3) * 255).to(torch.uint8)
    p = tmp_path / "x.png"
    Image.fromarray(img.numpy()).save(p)
    back = native().decode_png(p.read_bytes())
    assert torch.equal(back, img)


@pytest.fixture(scope="module")
def compiled(tmp_path_factory):
    root = tmp_path_factory.mktemp("src")
    write_synthetic_source(str(root), images=10, size=(96, 80), classes=3, seed=1)
    out = tmp_path_factory.mktemp("bin")
    stats = compile_split(str(root), str(out), "train", width=64, height=64)
    return root, stats


def test_compile_header_and_pixels(compiled):
    root, stats = compiled
    ds = CompiledDataset(stats["path"])
    assert len(ds) == 10 and ds.size == (64, 64)
    assert ds.class_names[1:] == ["class_1", "class_2", "class_3"]
    assert os.path.getsize(stats["path"]) == ds.header["total_size"]
    # pixels == area average with fractional coverage: 96x80 -> 64x64 equals nearest upsampling to
    # 192x320 (2x, 4x) followed by exact 3x5 block means
    import numpy as np
    from PIL import Image
    src = torch.from_numpy(np.array(Image.open(os.path.join(root, "train", "000001.png")).convert("RGB")))
    up = src.float().permute(2, 0, 1).repeat_interleave(4, 1).repeat_interleave(2, 2)
    ref = torch.nn.functional.avg_pool2d(up[None], (5, 3))[0] / 255
    assert (ds.image(0) - ref).abs().max() < 1.5 / 255


def test_compile_boxes_scaled(compiled):
    root, stats = compiled
    ds = CompiledDataset(stats["path"])
    for i in range(len(ds)):
        lines = [json.loads(l) for l in open(os.path.join(root, "train", f"{i + 1:06d}.jsonl")) if l.strip()]
        boxes, cls, _ = ds.instances(i)
        assert boxes.shape[0] == len(lines) - 0  # rectangles never vanish at this scale
        for b, rec in zip(boxes.tolist(), lines):
            x1, y1, x2, y2 = rec["bbox_xyxy"]
            exp = [round(x1 * 64 / 96), round(y1 * 64 / 80), round(x2 * 64 / 96), round(y2 * 64 / 80)]
            assert all(abs(a - e) <= 1 for a, e in zip(b, exp))


def test_loader_epoch_shard_and_targets(compiled):
    _, stats = compiled
    seen = []
    for rank in range(2):
        bl = BatchLoader(stats["path"], batch_size=2, shuffle=True, seed=3, shard_rank=rank, shard_count=2,
                         pixels="float32", max_targets=6)
        assert len(bl) == 2  # 5 batches -> 2 per rank
        for images, targets, idx in bl:
            assert images.shape == (2, 3, 64, 64)
            ds = bl.dataset
            for k, i in enumerate(idx):
                assert torch.equal(images[k], ds.image(i))
            assert targets.boxes.shape == (2, 6, 4)
            valid = targets.valid()
            assert (targets.boxes[valid] > 0).all() and (targets.boxes[valid] <= 1).all()
            seen += idx
    assert len(set(seen)) == len(seen) == 8


def test_loader_bf16_and_masks(compiled):
    _, stats = compiled
    bl = BatchLoader(stats["path"], batch_size=3, shuffle=False, pixels="bfloat16", max_targets=8, with_masks=True)
    images, targets, idx = next(iter(bl))
    assert images.dtype == torch.bfloat16
    assert (images.float() - torch.stack([bl.dataset.image(i) for i in idx])).abs().max() < 4e-3
    assert targets.masks.shape[0] == sum(targets.counts_host)


def test_compile_rejects_bad_sources(tmp_path):
    root = tmp_path / "bad"
    write_synthetic_source(str(root), splits=("train",), images=2)
    os.remove(root / "train" / "000002.jsonl")
    with pytest.raises(CompileError):
        compile_split(str(root), str(tmp_path / "o"), "train")
    cats = json.load(open(root / "categories.json"))
    cats["classes"].append({"id": 7, "name": "x"})
    json.dump(cats, open(root / "categories.json", "w"))
    with pytest.raises(CompileError):
        load_categories(str(root))
