"""Model zoo: the reference BlockDAR hybrid and the interleaved hybrid MoE LM."""
from .hybrid import HybridMoEModel, flax_path, count_params, active_params_per_token  # noqa: F401
from .moe import MoE  # noqa: F401
from .mixers import GatedDeltaNet2, Mamba2, MLA  # noqa: F401
