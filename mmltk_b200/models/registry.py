"""Model module registry and artifact requests.

A model family registers one :class:`ModelModule` (id, display name, presets with their
descriptors, capability flags, preset inference from an artifact path) in a
:class:`ModelRegistry`; the CLI and the inference runtime look families up by id, by preset
name or by artifact path.  :class:`ModelArtifactRequest` is what a caller asks to load: exactly
one of a weights file, an ONNX file or a TensorRT engine, plus an optional preset and
resolution.

Reference: `include/mmltk/model/module.h:12-54`, `src/model/module.cpp:23-68` (registry),
`include/mmltk/model/artifacts.h:17-52` (artifact request, exactly-one-input rule),
`src/rfdetr/core/module.cpp:16-74` (the RF-DETR module registered as ``"rfdetr"``).
"""
from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Dict, List, Optional

__all__ = ["ModelPresetDescriptor", "ModelModuleCapabilities", "ModelModule", "RfDetrModule", "ModelRegistry",
           "ModelArtifactRequest", "default_registry"]


@dataclass(frozen=True)
class ModelPresetDescriptor:
    module_id: str
    preset_name: str
    display_name: str
    size_label: str
    task: str
    canonical_weight_filename: str
    resolution: int


@dataclass(frozen=True)
class ModelModuleCapabilities:
    supports_weights: bool = False
    supports_onnx: bool = False
    supports_tensorrt: bool = False
    supports_training: bool = False
    supports_live: bool = False


class ModelModule:
    """One model family.  Subclasses provide the id, the presets and the capabilities."""

    module_id: str = ""
    display_name: str = ""

    def presets(self) -> List[ModelPresetDescriptor]:
        return []

    def owns_preset(self, preset_name: str) -> bool:
        return any(p.preset_name == preset_name for p in self.presets())

    def infer_preset_from_artifact_path(self, path: str) -> str:
        """Preset name implied by an artifact's file name ('' when nothing matches)."""
        return ""

    def capabilities(self) -> ModelModuleCapabilities:
        return ModelModuleCapabilities()


class RfDetrModule(ModelModule):
    """RF-DETR detection / segmentation (every preset of the catalog)."""

    module_id = "rfdetr"
    display_name = "RF-DETR"

    def presets(self) -> List[ModelPresetDescriptor]:
        from ..config.presets import PRESETS
        return [ModelPresetDescriptor(self.module_id, p.name, p.display_name, p.size_label, p.task,
                                      p.weight_filename, p.resolution) for p in PRESETS.values()]

    def owns_preset(self, preset_name: str) -> bool:
        from ..config.presets import find_preset
        return find_preset(preset_name) is not None

    def infer_preset_from_artifact_path(self, path: str) -> str:
        from ..config.presets import infer_preset_from_path
        spec = infer_preset_from_path(path)
        return spec.name if spec is not None else ""

    def capabilities(self) -> ModelModuleCapabilities:
        # ONNX export exists; running ONNX / TensorRT artifacts needs runtimes this image lacks
        return ModelModuleCapabilities(supports_weights=True, supports_onnx=False, supports_tensorrt=False,
                                       supports_training=True, supports_live=True)


class ModelRegistry:
    def __init__(self) -> None:
        self._modules: List[ModelModule] = []

    def register_module(self, module: ModelModule) -> None:
        if not module.module_id:
            raise ValueError("model module without an id")
        if self.find_module(module.module_id) is not None:
            raise ValueError(f"model module {module.module_id!r} is already registered")
        self._modules.append(module)

    def find_module(self, module_id: str) -> Optional[ModelModule]:
        return next((m for m in self._modules if m.module_id == module_id), None)

    def find_module_for_preset(self, preset_name: str) -> Optional[ModelModule]:
        return next((m for m in self._modules if m.owns_preset(preset_name)), None)

    def find_module_for_artifact_path(self, path: str) -> Optional[ModelModule]:
        return next((m for m in self._modules if m.infer_preset_from_artifact_path(path)), None)

    def presets(self) -> List[ModelPresetDescriptor]:
        return [p for m in self._modules for p in m.presets()]

    def empty(self) -> bool:
        return not self._modules

    def modules(self) -> List[ModelModule]:
        return list(self._modules)


_KINDS = ("weights", "onnx", "tensorrt")


@dataclass
class ModelArtifactRequest:
    """What to load: exactly one artifact (weights / ONNX / TensorRT), optional preset and
    resolution (0 = the preset's)."""
    weights_path: str = ""
    onnx_path: str = ""
    tensorrt_path: str = ""
    preset_name: str = ""
    resolution: int = 0

    def selected_input_count(self) -> int:
        return sum(1 for p in (self.weights_path, self.onnx_path, self.tensorrt_path) if p)

    def selected_input_kind(self) -> str:
        for kind, p in zip(_KINDS, (self.weights_path, self.onnx_path, self.tensorrt_path)):
            if p:
                return kind
        return "none"

    def input_path(self) -> str:
        return self.weights_path or self.onnx_path or self.tensorrt_path

    def validate(self) -> None:
        n = self.selected_input_count()
        if n > 1:
            raise ValueError("pass exactly one of --weights, --onnx, --tensorrt (got several)")
        if n == 0 and not self.preset_name:
            raise ValueError("pass one of --weights, --onnx, --tensorrt, or a --preset")
        if self.resolution < 0:
            raise ValueError("resolution must be positive")

    def resolve(self, registry: Optional["ModelRegistry"] = None) -> Dict[str, str]:
        """module id, preset name, input kind and paths (the reference's ``ResolvedModelArtifacts``)."""
        self.validate()
        reg = registry or default_registry()
        path = self.input_path()
        module = reg.find_module_for_preset(self.preset_name) if self.preset_name else None
        if module is None and path:
            module = reg.find_module_for_artifact_path(path)
        if module is None:
            raise ValueError(f"no model module owns preset {self.preset_name!r} or artifact {path!r}")
        preset = self.preset_name or module.infer_preset_from_artifact_path(path)
        out = {"module_id": module.module_id, "preset_name": preset, "input_kind": self.selected_input_kind(),
               "input_path": os.path.abspath(path) if path else "", "weights_path": "", "onnx_path": "",
               "tensorrt_path": "", "artifact_root": os.path.dirname(os.path.abspath(path)) if path else ""}
        if self.selected_input_kind() != "none":
            out[self.selected_input_kind() + "_path"] = out["input_path"]
        return out


_DEFAULT: List[ModelRegistry] = []


def default_registry() -> ModelRegistry:
    """The process-wide registry with every built-in model family registered."""
    if not _DEFAULT:
        reg = ModelRegistry()
        reg.register_module(RfDetrModule())
        _DEFAULT.append(reg)
    return _DEFAULT[0]
