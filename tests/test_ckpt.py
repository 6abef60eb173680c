"""Checkpoint formats: native archive round trip, upstream .pth bridge, loading
into a model (strict summary, encoder-head group expansion, class-count bridge)."""
import torch

from mmltk_b200.ckpt import (CheckpointMetadata, is_native_checkpoint, load_checkpoint, load_native_checkpoint,
                             load_weights, normalize_checkpoint, prepare_for_module, save_native_checkpoint,
                             write_upstream_checkpoint)
from mmltk_b200.ckpt.native import FORMAT
from mmltk_b200.models.rfdetr import build_model


def _tiny(**kw):
    torch.manual_seed(0)
    return build_model("rf-detr-tiny-test", **kw)


def test_native_roundtrip(tmp_path):
    sd = {"a.weight": torch.randn(3, 4).bfloat16(), "b.bias": torch.arange(5), "c": torch.ones(2, dtype=torch.bool)}
    meta = CheckpointMetadata("rf-detr-medium", "native", "/x", 91, {"ia_bce_loss": True, "focal_alpha": 0.25,
                                                                    "mask_point_sample_ratio": 16})
    p = str(tmp_path / "c.pt")
    save_native_checkpoint(p, sd, meta, extra={"epoch": 3, "lr_scheduler": "step"})
    assert is_native_checkpoint(p)
    ck = load_native_checkpoint(p)
    assert list(ck.state_dict) == list(sd)
    for k in sd:
        assert torch.equal(ck.state_dict[k], sd[k]) and ck.state_dict[k].dtype == sd[k].dtype
    assert ck.metadata.preset_name == "rf-detr-medium" and ck.metadata.num_classes == 91
    assert ck.metadata.optional == {"ia_bce_loss": True, "focal_alpha": 0.25, "mask_point_sample_ratio": 16}
    assert ck.extra == {"epoch": 3, "lr_scheduler": "step"}
    # the container is a libtorch archive: TorchScript can open it too
    m = torch.jit.load(p)
    assert m.format == FORMAT and m.state.entry_000000.name == "a.weight"


def test_upstream_bridge(tmp_path):
    model = _tiny()
    p = str(tmp_path / "rf-detr-medium.pth")
    write_upstream_checkpoint(p, model.state_dict(), {"ia_bce_loss": True, "set_cost_class": 2, "junk": "x"})
    assert not is_native_checkpoint(p)
    ck = load_checkpoint(p)
    assert ck.metadata.source_kind == "upstream-python"
    assert ck.metadata.optional == {"ia_bce_loss": True, "set_cost_class": 2.0}
    assert ck.metadata.num_classes == model.class_embed.weight.shape[0]
    out = str(tmp_path / "n.pt")
    normalize_checkpoint(p, out)
    assert is_native_checkpoint(out)
    m2 = _tiny()
    s = load_weights(m2, out)
    assert s.ok()
    for k, v in model.state_dict().items():
        assert torch.equal(v, m2.state_dict()[k]), k


def test_encoder_group_expansion_and_query_narrowing():
    model = _tiny(group_detr=3)
    target = model.state_dict()
    enc = [k for k in target if k.startswith("transformer.enc_out_class_embed.")]
    assert any(".2." in k for k in enc)
    src = {k[len("transformer."):]: torch.full_like(v, 7.0) for k, v in target.items()
           if k.startswith("transformer.enc_out_class_embed.0.")}
    q = target["query_feat.weight"]
    src["query_feat.weight"] = torch.zeros(q.shape[0] + 5, q.shape[1])
    prep = prepare_for_module(src, target)
    for g in range(3):
        assert torch.all(prep[f"transformer.enc_out_class_embed.{g}.weight"] == 7.0)
    assert prep["query_feat.weight"].shape == q.shape


def test_class_count_bridge_repeats_rows():
    src = _tiny(num_classes=4)
    dst = _tiny(num_classes=10)
    s = load_weights(dst, _as_ckpt(src))
    assert s.ok()
    w_src = src.class_embed.weight
    w_dst = dst.class_embed.weight
    assert w_dst.shape[0] == 10
    for r in range(10):
        assert torch.equal(w_dst[r], w_src[r % 4])
    assert torch.equal(dst.bbox_embed.layers[0].weight, src.bbox_embed.layers[0].weight)


def test_strict_summary_reports_mismatch():
    m = _tiny()
    sd = dict(m.state_dict())
    sd.pop("class_embed.bias")
    sd["bogus"] = torch.zeros(1)
    from mmltk_b200.ckpt import apply_to_module
    s = apply_to_module(m, sd, strict=False)
    assert s.missing == ["class_embed.bias"] and s.unexpected == ["bogus"]
    try:
        apply_to_module(m, sd, strict=True)
        raise AssertionError("strict load must fail")
    except RuntimeError as e:
        assert "bogus" in str(e)


def _as_ckpt(model):
    from mmltk_b200.ckpt.native import NativeCheckpoint
    return NativeCheckpoint(CheckpointMetadata(num_classes=model.class_embed.weight.shape[0]),
                            dict(model.state_dict()))
