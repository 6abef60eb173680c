"""Inference: fused post-process, CUDA-graph predictor, prediction / evaluation workflows."""
from .postprocess import postprocess, postprocess_reference
from .predictor import Predictor, encode_mask_rle, evaluate_compiled, predict_compiled, predict_images, \
    resolve_model, write_predictions_json

__all__ = ["postprocess", "postprocess_reference", "Predictor", "encode_mask_rle", "evaluate_compiled",
           "predict_compiled", "predict_images", "resolve_model", "write_predictions_json"]
