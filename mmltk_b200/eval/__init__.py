"""Evaluation: COCO-style AP over compiled splits."""
from .coco import CocoEvaluator

__all__ = ["CocoEvaluator"]
