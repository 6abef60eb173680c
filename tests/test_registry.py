"""Model module registry and artifact requests (reference `tests/core/model_registry.test.cpp`
semantics: lookup by id / preset / artifact path, duplicate ids rejected, exactly one artifact)."""
import json

import pytest

from mmltk_b200.models.registry import (ModelArtifactRequest, ModelModule, ModelRegistry, RfDetrModule,
                                        default_registry)


def test_default_registry_finds_rfdetr_by_id_preset_and_path():
    reg = default_registry()
    assert not reg.empty()
    m = reg.find_module("rfdetr")
    assert isinstance(m, RfDetrModule)
    assert reg.find_module_for_preset("rf-detr-medium") is m
    assert reg.find_module_for_preset("no-such-preset") is None
    assert reg.find_module_for_artifact_path("/x/rf-detr-medium.pth") is m
    names = {p.preset_name for p in reg.presets()}
    assert {"rf-detr-nano", "rf-detr-medium", "rf-detr-seg-small"} <= names
    caps = m.capabilities()
    assert caps.supports_weights and caps.supports_training and not caps.supports_tensorrt


def test_duplicate_module_id_is_rejected():
    reg = ModelRegistry()
    reg.register_module(RfDetrModule())
    with pytest.raises(ValueError):
        reg.register_module(RfDetrModule())
    with pytest.raises(ValueError):
        reg.register_module(ModelModule())


def test_artifact_request_exactly_one_input():
    assert ModelArtifactRequest(weights_path="a.pth").selected_input_kind() == "weights"
    assert ModelArtifactRequest(onnx_path="a.onnx").selected_input_kind() == "onnx"
    assert ModelArtifactRequest(preset_name="rf-detr-nano").selected_input_kind() == "none"
    with pytest.raises(ValueError):
        ModelArtifactRequest(weights_path="a.pth", onnx_path="a.onnx").validate()
    with pytest.raises(ValueError):
        ModelArtifactRequest().validate()
    r = ModelArtifactRequest(weights_path="/w/rf-detr-small.pth").resolve()
    assert r["module_id"] == "rfdetr" and r["preset_name"] == "rf-detr-small" and r["input_kind"] == "weights"
    assert r["weights_path"] == "/w/rf-detr-small.pth"


def test_cli_models_lists_the_registry(capsys):
    from mmltk_b200.cli.main import main
    assert main(["models"]) == 0
    out = json.loads(capsys.readouterr().out)
    assert out[0]["module_id"] == "rfdetr" and out[0]["presets"]
