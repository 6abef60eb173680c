"""Model export: ONNX (opset 19) and ONNX model inspection."""
from .onnx import export_onnx, onnx_info

__all__ = ["export_onnx", "onnx_info"]
