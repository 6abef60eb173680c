"""Headless live analysis: frame sources, a latest-frame lease ring between capture and
analysis, GPU letterbox -> CUDA-graph predictor -> on-device drawing."""
from .analyzer import FrameAnalyzer, LiveStats, run_live
from .source import SyntheticFrameSource

__all__ = ["FrameAnalyzer", "LiveStats", "run_live", "SyntheticFrameSource"]
