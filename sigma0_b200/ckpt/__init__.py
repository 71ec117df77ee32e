"""Checkpoints: flat-buffer save/restore in the reference's step-directory layout, and the
Orbax StandardSave layout (zarr v2) read and written without Orbax."""
from .checkpoint import CheckpointManager, CheckpointError, flax_path, remap_step
from .orbax import OrbaxFormatError, read_standard_item, write_step

__all__ = ["CheckpointManager", "CheckpointError", "flax_path", "remap_step", "OrbaxFormatError",
           "read_standard_item", "write_step"]
