"""Inference: post-process kernel vs torch statement, predictor + JSON records,
evaluation workflow, checkpoint -> predictor resolution."""
import json
import os

import pytest
import torch

from mmltk_b200.ckpt import CheckpointMetadata, save_native_checkpoint
from mmltk_b200.data.compiler import compile_split
from mmltk_b200.data.source import write_synthetic_source
from mmltk_b200.infer import (Predictor, encode_mask_rle, evaluate_compiled, postprocess_reference, predict_compiled,
                              resolve_model, write_predictions_json)
from mmltk_b200.models.rfdetr import build_model


def test_postprocess_reference_semantics():
    torch.manual_seed(0)
    logits = torch.randn(2, 5, 3)
    logits[0, 1, 2] = logits[0, 3, 0] = 9.0           # tie: lower flat index (5) first, then 9
    boxes = torch.rand(2, 5, 4)
    r = postprocess_reference(logits, boxes, 4, (10, 20))
    assert r["queries"][0, 0] == 1 and r["labels"][0, 0] == 2
    assert r["queries"][0, 1] == 3 and r["labels"][0, 1] == 0
    assert torch.allclose(r["scores"][0, 0], torch.sigmoid(torch.tensor(9.0)))
    cx, cy, w, h = boxes[0, 1]
    assert torch.allclose(r["boxes"][0, 0], torch.stack([(cx - w / 2) * 20, (cy - h / 2) * 10,
                                                         (cx + w / 2) * 20, (cy + h / 2) * 10]))


def test_mask_rle():
    m = torch.zeros(3, 4, dtype=torch.bool)
    m[0, 1:3] = True
    m[1, 3] = m[2, 0] = True
    assert encode_mask_rle(m) == "1:2 7:2"


@pytest.fixture(scope="module")
def compiled32(tmp_path_factory):
    root = tmp_path_factory.mktemp("isrc")
    write_synthetic_source(str(root), splits=("val",), images=5, size=(48, 40), classes=3, seed=3)
    st = compile_split(str(root), str(tmp_path_factory.mktemp("ibin")), "val", width=32, height=32)
    return st["path"]


def test_predict_and_evaluate_cpu(compiled32, tmp_path):
    torch.manual_seed(0)
    model = build_model("rf-detr-tiny-test", num_classes=4)
    p = Predictor(model, device="cpu")
    recs, timing = predict_compiled(p, compiled32, batch_size=2, threshold=0.0)
    assert len(recs) == 5 and timing["images"] == 5
    assert all(len(r["detections"]) == model.cfg.num_select for r in recs)
    d = recs[0]["detections"][0]
    assert set(d) == {"label", "score", "xyxy"} and recs[0]["image_id"] == recs[0]["dataset_index"] + 1
    out = str(tmp_path / "pred.json")
    write_predictions_json(out, recs, {"preset_name": "rf-detr-tiny-test"}, "compiled_dataset", compiled_path=compiled32)
    js = json.load(open(out))
    assert js["mask_rle_encoding"] == "row_major_start_length" and len(js["records"]) == 5
    ev = evaluate_compiled(p, compiled32, batch_size=2)
    assert ev["images"] == 5 and 0.0 <= ev["bbox"]["ap"] <= 1.0


def test_resolve_model_from_checkpoint(tmp_path):
    m = build_model("rf-detr-tiny-test", num_classes=6)
    path = str(tmp_path / "w.pt")
    save_native_checkpoint(path, m.state_dict(), CheckpointMetadata("rf-detr-tiny-test", num_classes=6))
    m2, info = resolve_model(path)
    assert info["preset_name"] == "rf-detr-tiny-test" and m2.class_embed.weight.shape[0] == 6
    for k, v in m.state_dict().items():
        assert torch.equal(v, m2.state_dict()[k])


@pytest.mark.gpu
def test_topk_kernel_matches_reference():
    from mmltk_b200.ops import kernels
    torch.manual_seed(1)
    for (B, Q, C, K, dt) in [(2, 300, 91, 300, torch.float32), (3, 100, 7, 100, torch.bfloat16),
                             (1, 17, 5, 85, torch.float32)]:
        logits = torch.randn(B, Q, C, device="cuda").to(dt)
        logits[0, 3, :] = 1.0                                  # ties
        boxes = torch.rand(B, Q, 4, device="cuda")
        s, l, b, q = kernels().topk_postprocess(logits, boxes, K, None, 432.0, 576.0)
        r = postprocess_reference(logits.cpu(), boxes.cpu(), K, (432, 576))
        assert torch.equal(q.cpu(), r["queries"]) and torch.equal(l.cpu(), r["labels"])
        assert torch.allclose(s.cpu(), r["scores"], atol=1e-6)
        assert torch.allclose(b.cpu(), r["boxes"], atol=1e-3)


@pytest.mark.gpu
def test_graph_predictor_matches_eager(compiled32):
    torch.manual_seed(0)
    model = build_model("rf-detr-tiny-test", num_classes=4)
    eager = Predictor(model, device="cuda", cuda_graph=False)
    graph = Predictor(build_model("rf-detr-tiny-test", num_classes=4), device="cuda", cuda_graph=True)
    graph.model.load_state_dict(eager.model.state_dict())
    x = torch.randint(0, 256, (2, 3, 32, 32), dtype=torch.uint8)
    a = eager(x.cuda())
    for _ in range(2):
        g = graph(x.cuda())
    torch.cuda.synchronize()
    assert torch.equal(a["queries"], g["queries"])
    assert torch.allclose(a["boxes"], g["boxes"], atol=1e-3)
    host = graph.predict_host(x)                  # one packed device-to-host copy
    for k, v in g.items():
        if k != "masks":
            assert not host[k].is_cuda and host[k].dtype == v.dtype and torch.equal(host[k], v.cpu()), k
    lat = graph.latency(iters=20, warmup=3, batch=1)
    assert lat["p50_ms"] > 0
    assert graph.latency(iters=5, warmup=1, batch=1, pin_cpus=False)["p50_ms"] > 0
    graph.release()


def test_validate_native_vs_export_report(compiled32):
    """validate: both backends scored on the same images with the reference's report keys; on
    the CPU the native predictor runs the same fp32 statement as the export graph, so the two agree."""
    from mmltk_b200.infer.validate import validate_compiled
    torch.manual_seed(0)
    model = build_model("rf-detr-tiny-test", num_classes=4)
    rep = validate_compiled(model, compiled32, ("native", "export"), batch_size=2, limit=4, device="cpu")
    assert rep["eval_order"] == ["native", "export"] and rep["images"] == 4
    for name in ("native", "export"):
        assert 0.0 <= rep[name]["bbox_ap"] <= 1.0 and rep[name]["img_per_s"] > 0
    al = rep["alignment_probe"]
    assert al["images_compared"] == 4
    assert al["top1_score_abs_diff_max"] < 1e-4 and al["top1_box_abs_diff_px_max"] < 1e-2
    assert abs(rep["delta_export_minus_native"]["bbox_ap"]) < 1e-9


@pytest.mark.gpu
def test_validate_gpu_predictor_against_export_graph(compiled32, cuda_device):
    """The bf16 B200 predictor against the fp32 export graph: same images, close top-1 detections."""
    from mmltk_b200.infer.validate import validate_compiled
    torch.manual_seed(0)
    model = build_model("rf-detr-tiny-test", num_classes=4)
    rep = validate_compiled(model, compiled32, ("native", "export"), batch_size=1, limit=5, device=cuda_device)
    assert rep["images"] == 5 and rep["alignment_probe"]["images_compared"] == 5
    assert rep["alignment_probe"]["top1_score_abs_diff_mean"] < 0.05
