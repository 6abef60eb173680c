"""Checkpoints: native archives, upstream ``.pth`` files, loading into a model, resume state."""
from .apply import LoadSummary, apply_to_module, checkpoint_class_count, load_checkpoint, load_weights, \
    normalize_checkpoint, prepare_for_module
from .native import CheckpointMetadata, NativeCheckpoint, is_native_checkpoint, load_native_checkpoint, \
    save_native_checkpoint
from .upstream import load_upstream_checkpoint, write_upstream_checkpoint

__all__ = ["LoadSummary", "apply_to_module", "checkpoint_class_count", "load_checkpoint", "load_weights",
           "normalize_checkpoint", "prepare_for_module", "CheckpointMetadata", "NativeCheckpoint",
           "is_native_checkpoint", "load_native_checkpoint", "save_native_checkpoint", "load_upstream_checkpoint",
           "write_upstream_checkpoint"]
