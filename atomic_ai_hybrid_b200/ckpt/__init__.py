"""Checkpoints in the reference's parameter-tree layout (safetensors, sharded, async)."""
from .manager import CheckpointManager, make_manager, reference_dtype, upload_slot, download_slot, SLOTS  # noqa: F401
from .safetensors_io import save_file, load_file  # noqa: F401
