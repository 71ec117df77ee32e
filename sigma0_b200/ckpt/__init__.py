"""Checkpoints: flat-buffer save/restore in the reference's step-directory layout."""
from .checkpoint import CheckpointManager, CheckpointError, flax_path, remap_step

__all__ = ["CheckpointManager", "CheckpointError", "flax_path", "remap_step"]
