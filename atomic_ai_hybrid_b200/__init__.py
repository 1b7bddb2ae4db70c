"""atomic_ai_hybrid_b200: a Blackwell (sm_100a) native training framework for
hybrid GatedDeltaNet-2 / Mamba2 / MoE language models."""
from .config import ModelConfig, get_preset, PRESETS  # noqa: F401

__version__ = "0.1.0"
