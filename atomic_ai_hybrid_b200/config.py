"""Model configuration and named presets.

`ModelConfig` keeps every field name of the reference's frozen dataclass
(reference `model.py:220-256`) so that code written against the reference reads
the same here.  Extra fields carry what the reference hard-codes or lacks:

* ``arch``            -- ``"blockdar"`` (the reference stack: blocks of
                          ``layers_per_block`` sublayers with DAR / intra-block
                          source attention and one MoE per block) or
                          ``"interleaved"`` (each sublayer followed by its own MoE,
                          no DAR; the layout of the benchmark configs).
* ``ffn_act``         -- ``"gelu"`` (reference experts, tanh-approx GELU) or
                          ``"swiglu"``.
* ``n_shared_experts`` / ``n_routed_experts`` -- the reference counts its one
                          shared expert inside ``num_experts`` (``E_routed =
                          num_experts - 1``, reference `atomic_ops/moe_gmm.py:388`);
                          ``n_routed_experts=None`` keeps that convention.
* ``expand`` / ``n_heads_ssm`` give Mamba2 ``d_inner = d_model*expand`` split in
  ``n_heads_ssm`` heads, as in the reference.
* ``gdn_chunk`` / ``ssd_chunk`` -- chunk lengths of the chunked scans
  (reference: GDN ``BT=256`` in `atomic_ops/kernel_a_scores.py:15`, Mamba2
  ``deltanet_chunk_size``).  The results do not depend on the chunk length
  beyond rounding.
"""
from __future__ import annotations

import dataclasses
from dataclasses import dataclass, field
from typing import Optional, Tuple

REFERENCE_LAYER_TYPES: Tuple[str, ...] = (
    "gdn2", "gdn2", "mla",
    "gdn2", "mamba2", "gdn2",
    "gdn2", "gdn2", "gdn2",
    "gdn2", "gdn2", "mla",
    "gdn2", "mamba2", "gdn2",
    "gdn2", "gdn2", "gdn2",
    "gdn2", "gdn2", "mla",
)


@dataclass(frozen=True)
class ModelConfig:
    d_model: int = 768
    d_state: int = 128
    d_conv: int = 4
    expand: int = 2
    n_heads: int = 8
    n_heads_ssm: int = 8
    d_latent: int = 384
    d_ff: int = 3072
    num_experts: int = 8
    top_k: int = 2
    num_layers: int = 21
    layers_per_block: int = 3
    vocab_size: int = 151936
    dropout_rate: float = 0.1
    router_aux_loss_coef: float = 0.01
    router_z_loss_coef: float = 0.0001
    moe_capacity_factor: float = 1.25
    tie_embeddings: bool = True
    label_smoothing: float = 0.05
    router_noise_std: float = 0.3
    use_flash_attention: bool = True
    deltanet_chunk_size: int = 256
    layer_types: Tuple[str, ...] = REFERENCE_LAYER_TYPES

    # ---- fields this framework adds -------------------------------------
    arch: str = "blockdar"
    ffn_act: str = "gelu"
    n_shared_experts: int = 1
    n_routed_experts: Optional[int] = None
    gdn_chunk: int = 64
    ssd_chunk: int = 64
    init_std: float = 0.02
    # "reference": A_log ~ U[0,1), dt_proj bias 0 (reference initialisers);
    # "mamba": A_log ~ U[log 1, log 16], dt bias = softplus^-1(U[1e-3, 0.1]).
    ssm_init: str = "reference"
    tie_lm_head: bool = True

    @property
    def e_routed(self) -> int:
        if self.n_routed_experts is not None:
            return self.n_routed_experts
        return self.num_experts - self.n_shared_experts

    @property
    def d_inner(self) -> int:
        return self.d_model * self.expand

    @property
    def ssm_headdim(self) -> int:
        return self.d_inner // self.n_heads_ssm

    @property
    def d_head(self) -> int:
        return self.d_model // self.n_heads

    @property
    def num_blocks(self) -> int:
        return self.num_layers // self.layers_per_block

    def replace(self, **kw) -> "ModelConfig":
        return dataclasses.replace(self, **kw)

    def validate(self) -> None:
        assert len(self.layer_types) >= self.num_layers, "layer_types shorter than num_layers"
        assert self.d_model % self.n_heads == 0
        assert self.d_inner % self.n_heads_ssm == 0
        assert self.e_routed >= self.top_k
        assert self.arch in ("blockdar", "interleaved")
        assert self.ffn_act in ("gelu", "swiglu")
        if self.arch == "blockdar":
            assert self.num_layers % self.layers_per_block == 0


def _alternating(n: int, first: str = "mamba2", second: str = "gdn2") -> Tuple[str, ...]:
    return tuple(first if i % 2 == 0 else second for i in range(n))


def _pattern_3to1(n: int) -> Tuple[str, ...]:
    return tuple("mamba2" if i % 4 == 3 else "gdn2" for i in range(n))


# Reference defaults, exactly `ModelConfig()` of the reference.
REFERENCE_DEFAULT = ModelConfig()

# The configuration the reference's train.py trains (reference `train.py:405-436`, the same
# in `traivn.py:303-334`): d_model 768, 6 heads, d_latent 768, 24 layers in blocks of 3 with
# MLA every third layer of blocks 0, 2, 4, 6, vocab 128256 with tied embeddings, aux 0.03,
# z 3e-4, no label smoothing, router noise 0.1; fields it does not set keep the ModelConfig
# defaults (n_heads_ssm 8, dropout 0.1, ...).
REFERENCE_TRAIN_LAYER_TYPES: Tuple[str, ...] = (
    "gdn2", "gdn2", "mla",
    "gdn2", "mamba2", "gdn2",
    "gdn2", "gdn2", "mla",
    "gdn2", "mamba2", "gdn2",
    "gdn2", "gdn2", "mla",
    "gdn2", "mamba2", "gdn2",
    "gdn2", "gdn2", "mla",
    "gdn2", "gdn2", "gdn2",
)
REFERENCE_TRAIN = ModelConfig(
    d_model=768, d_state=128, d_conv=4, expand=2, n_heads=6, d_latent=768, d_ff=4096,
    num_experts=8, top_k=2, moe_capacity_factor=1.25, router_aux_loss_coef=0.03,
    router_z_loss_coef=0.0003, num_layers=24, layers_per_block=3, vocab_size=128256,
    tie_embeddings=True, label_smoothing=0.0, router_noise_std=0.1, use_flash_attention=True,
    deltanet_chunk_size=256, layer_types=REFERENCE_TRAIN_LAYER_TYPES,
)

# Config 1 of the benchmark spec: tiny CPU model, fp32 parity.
TINY = ModelConfig(
    d_model=256, d_state=64, d_conv=4, expand=1, n_heads=4, n_heads_ssm=4,
    d_latent=128, d_ff=512, num_experts=8, top_k=2, num_layers=4,
    layers_per_block=1, vocab_size=4096, layer_types=_alternating(4),
    arch="interleaved", ffn_act="swiglu", n_shared_experts=0, n_routed_experts=8,
    gdn_chunk=64, ssd_chunk=64, deltanet_chunk_size=64, ssm_init="mamba",
    dropout_rate=0.0, router_noise_std=0.0,
)

# Config 3: hybrid MoE LM, d_model 2048, 24 layers alternating GDN (16x128) and
# Mamba2 (32x64, d_state 128); 32 routed experts top-4 of hidden 1024 + 1 shared.
HYBRID_1B = ModelConfig(
    d_model=2048, d_state=128, d_conv=4, expand=1, n_heads=16, n_heads_ssm=32,
    d_latent=512, d_ff=1024, num_experts=33, top_k=4, num_layers=24,
    layers_per_block=1, vocab_size=50304, layer_types=_alternating(24, "gdn2", "mamba2"),
    arch="interleaved", ffn_act="swiglu", n_shared_experts=1, n_routed_experts=32,
    gdn_chunk=64, ssd_chunk=64, deltanet_chunk_size=64, ssm_init="mamba",
    dropout_rate=0.0,
)

# Config 4: 7B-total / 1.3B-active, 3 GDN : 1 Mamba2, 64 experts top-6 of 1536.
HYBRID_7B = ModelConfig(
    d_model=3072, d_state=128, d_conv=4, expand=1, n_heads=24, n_heads_ssm=48,
    d_latent=768, d_ff=1536, num_experts=65, top_k=6, num_layers=32,
    layers_per_block=1, vocab_size=50304, layer_types=_pattern_3to1(32),
    arch="interleaved", ffn_act="swiglu", n_shared_experts=1, n_routed_experts=64,
    gdn_chunk=64, ssd_chunk=64, deltanet_chunk_size=64, ssm_init="mamba",
    dropout_rate=0.0,
)

# Config 5: long context, TP=8.
HYBRID_LONG = ModelConfig(
    d_model=4096, d_state=128, d_conv=4, expand=1, n_heads=32, n_heads_ssm=64,
    d_latent=1024, d_ff=2048, num_experts=65, top_k=8, num_layers=48,
    layers_per_block=1, vocab_size=50304, layer_types=_alternating(48, "gdn2", "mamba2"),
    arch="interleaved", ffn_act="swiglu", n_shared_experts=1, n_routed_experts=64,
    gdn_chunk=64, ssd_chunk=64, deltanet_chunk_size=64, ssm_init="mamba",
    dropout_rate=0.0,
)

# Small BlockDAR model with every sublayer kind; used by tests of the reference stack.
REFERENCE_TINY = ModelConfig(
    d_model=128, d_state=32, d_conv=4, expand=2, n_heads=2, n_heads_ssm=4,
    d_latent=64, d_ff=256, num_experts=5, top_k=2, num_layers=6, layers_per_block=3,
    vocab_size=512, layer_types=("gdn2", "mamba2", "mla", "gdn2", "gdn2", "mamba2"),
    deltanet_chunk_size=64, gdn_chunk=64, ssd_chunk=64,
)

PRESETS = {
    "reference": REFERENCE_TRAIN,
    "reference_default": REFERENCE_DEFAULT,
    "reference_tiny": REFERENCE_TINY,
    "tiny": TINY,
    "hybrid_1b": HYBRID_1B,
    "hybrid_7b": HYBRID_7B,
    "hybrid_long": HYBRID_LONG,
}


def get_preset(name: str, **overrides) -> ModelConfig:
    cfg = PRESETS[name]
    if overrides:
        cfg = cfg.replace(**overrides)
    cfg.validate()
    return cfg


def load_yaml_config(path: str) -> ModelConfig:
    """Read a YAML file ``{preset: name, overrides: {...}}`` or a flat field map."""
    import yaml

    with open(path) as f:
        data = yaml.safe_load(f) or {}
    data.pop("train", None)  # the run settings of a configuration file (train.py)
    if "preset" in data:
        over = dict(data.get("overrides") or {})
    else:
        over, data = dict(data), {"preset": "reference_default"}
    if "layer_types" in over:
        over["layer_types"] = tuple(over["layer_types"])
    return get_preset(data["preset"], **over)
