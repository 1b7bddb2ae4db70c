"""Full language models.

``HybridMoEModel`` builds either layout selected by ``cfg.arch``:

* ``"blockdar"`` -- the reference ``FullHybridMoEModel`` (`model.py:906-952`):
  blocks of ``layers_per_block`` sublayers (``gdn2``/``mamba2``/``mla``) whose
  input is an intra-block source-softmax mix of the block input and the deltas
  of the earlier sublayers (``IntraBlockAttention``, `model.py:707-734`), residual
  clips of ``+-5e2`` after Mamba2 and ``+-1e3`` otherwise, then ``norm_2`` and one
  MoE per block.  ``HybridDARAttention`` parameters exist as in the reference.
  The reference adds the DAR output to a local ``current_x`` that nothing reads
  afterwards (`model.py:798-826`), so its value never reaches the output; the
  module therefore skips that computation unless ``compute_dar=True``.
* ``"interleaved"`` -- pre-norm residual stack where every sublayer is followed by
  its own MoE (the benchmark configurations).

Parameter names equal the flax paths with ``/`` replaced by ``.``
(``block_0.layer_1.sublayer.gdn2.q_proj.kernel``).
"""
from __future__ import annotations

import math
from typing import Dict, List, Optional

import torch
import torch.nn as nn

from .. import ops
from ..config import ModelConfig
from ..ops import reference as R
from ..parallel.cp import get_cp
from ..parallel.tp import get_tp
from ..utils.diag import DIAG
from ..utils.nvtx import nvtx_range
from .layers import Dense, RMSNorm
from .mixers import MLA, GatedDeltaNet2, Mamba2
from .moe import MoE


class IntraBlockAttention(nn.Module):
    def __init__(self, cfg: ModelConfig, n_sources: int):
        super().__init__()
        self.n = n_sources
        self.d_latent = cfg.d_latent
        if n_sources > 1:
            self.q_proj = Dense(cfg.d_model, cfg.d_latent)
            for i in range(n_sources):
                setattr(self, f"k_proj_{i}", Dense(cfg.d_model, cfg.d_latent))

    def forward(self, sources: List[torch.Tensor], block_input: torch.Tensor) -> torch.Tensor:
        if len(sources) == 1:
            return sources[0]
        q = self.q_proj(block_input)
        scale = 1.0 / math.sqrt(self.d_latent)
        if ops.use_cuda(q):
            from ..ops import kernels as K
            ks = [getattr(self, f"k_proj_{i}")(s) for i, s in enumerate(sources)]
            out = K.source_mix(q, ks, sources, scale)
            if out is not None:
                return out
        scores = torch.stack([(q * getattr(self, f"k_proj_{i}")(s)).sum(-1) for i, s in enumerate(sources)], 0)
        wts = torch.softmax(scores.float() * scale, 0).to(block_input.dtype)
        mixed = sum(wts[i][..., None] * s for i, s in enumerate(sources))
        return mixed.to(block_input.dtype)


class HybridDARAttention(nn.Module):
    def __init__(self, cfg: ModelConfig, n_sources: int):
        super().__init__()
        self.n = n_sources
        self.d_latent = cfg.d_latent
        if n_sources > 0:
            self.k_proj = Dense(cfg.d_model, cfg.d_latent)
            self.q_proj = Dense(cfg.d_model, cfg.d_latent)

    def forward(self, current_x, sources):
        if len(sources) == 0:
            return torch.zeros_like(current_x)
        q = self.q_proj(current_x)
        if ops.use_cuda(q):
            from ..ops import kernels as K
            out = K.source_mix(q, [self.k_proj(s) for s in sources], sources, 1.0 / math.sqrt(self.d_latent))
            if out is not None:
                return out
        scores = torch.stack([(q * self.k_proj(s)).sum(-1) for s in sources], 0) / math.sqrt(self.d_latent)
        wts = torch.softmax(scores.float(), 0).to(current_x.dtype)
        return sum(wts[i][..., None] * s for i, s in enumerate(sources)).to(current_x.dtype)


class Sublayer(nn.Module):
    def __init__(self, cfg: ModelConfig, layer_type: str):
        super().__init__()
        self.layer_type = layer_type
        if layer_type == "gdn2":
            self.gdn2 = GatedDeltaNet2(cfg)
        elif layer_type == "mamba2":
            self.mamba2 = Mamba2(cfg)
        elif layer_type == "mla":
            self.mla = MLA(cfg)
        else:
            raise ValueError(f"Unknown layer_type: {layer_type}")

    def forward(self, x, cos=None, sin=None):
        if self.layer_type == "gdn2":
            return self.gdn2(x)
        if self.layer_type == "mamba2":
            return self.mamba2(x)
        return self.mla(x, cos, sin)


class BlockDARLayer(nn.Module):
    def __init__(self, cfg: ModelConfig, layer_type: str, block_idx: int, pos_in_block: int, compute_dar: bool):
        super().__init__()
        self.layer_type = layer_type
        self.compute_dar = compute_dar
        n_dar = block_idx + pos_in_block
        self.dar = HybridDARAttention(cfg, n_dar)
        self.intra = IntraBlockAttention(cfg, 1 + pos_in_block)
        self.pre_sublayer_norm = RMSNorm(cfg.d_model)
        self.sublayer = Sublayer(cfg, layer_type)

    def forward(self, current_x, block_input, local_deltas, history, cos, sin):
        if self.compute_dar:
            _ = current_x + self.dar(current_x, list(history) + list(local_deltas))
        mixed = self.intra([block_input] + list(local_deltas), block_input)
        mixed = self.pre_sublayer_norm(mixed)
        delta = self.sublayer(mixed, cos, sin)
        delta = ops.grad_sanitize(delta)
        return ops.sanitize(delta, 1e3)


class BlockDAR(nn.Module):
    def __init__(self, cfg: ModelConfig, block_idx: int, compute_dar: bool):
        super().__init__()
        self.cfg = cfg
        self.block_idx = block_idx
        lpb = cfg.layers_per_block
        self.layer_ids = [block_idx * lpb + i for i in range(lpb)]
        for i, li in enumerate(self.layer_ids):
            setattr(self, f"layer_{li}", BlockDARLayer(cfg, cfg.layer_types[li], block_idx, i, compute_dar))
        self.norm_2 = RMSNorm(cfg.d_model)
        self.moe = MoE(cfg)

    def forward(self, current_x, history: List[torch.Tensor], cos, sin, stats: List[Dict]):
        block_input = current_x
        local: List[torch.Tensor] = []
        for li in self.layer_ids:
            layer = getattr(self, f"layer_{li}")
            delta = layer(current_x, block_input, local, history, cos, sin)
            tag = f"block={self.block_idx} layer={li} type={layer.layer_type}"
            DIAG.nonfinite(f"delta: {tag}", delta)
            DIAG.resid_breakdown(tag, current_x, delta)
            local.append(delta)
            clip = 5e2 if layer.layer_type == "mamba2" else 1e3
            summed = current_x + delta
            DIAG.maxabs(tag, summed)
            current_x = ops.sanitize(summed, clip)
        history.append(sum(local))
        st: Dict[str, torch.Tensor] = {}
        moe_out = self.moe(self.norm_2(current_x), st)
        DIAG.nonfinite(f"moe_out: block={self.block_idx}", moe_out)
        stats.append(st)
        return ops.sanitize(current_x + moe_out, 1e3)


class InterleavedLayer(nn.Module):
    """``x += sublayer(pre_norm(x))``; ``x += moe(norm_2(x))`` with the reference's
    residual clip values."""

    def __init__(self, cfg: ModelConfig, layer_type: str):
        super().__init__()
        self.layer_type = layer_type
        self.pre_norm = RMSNorm(cfg.d_model)
        self.sublayer = Sublayer(cfg, layer_type)
        self.norm_2 = RMSNorm(cfg.d_model)
        self.moe = MoE(cfg)

    def _tag(self) -> str:
        return f"layer={getattr(self, 'layer_idx', '?')} type={self.layer_type}"

    def forward(self, x, cos, sin, stats: List[Dict]):
        tag = self._tag()
        delta = ops.grad_sanitize(self.sublayer(self.pre_norm(x), cos, sin), tag=f"sublayer {tag}")
        DIAG.nonfinite(f"delta: {tag}", delta)
        DIAG.resid_breakdown(tag, x, delta)
        clip = 5e2 if self.layer_type == "mamba2" else 1e3
        summed = x + delta
        DIAG.maxabs(tag, summed)
        x = ops.sanitize(summed, clip)
        st: Dict[str, torch.Tensor] = {}
        m = self.moe(self.norm_2(x), st)
        DIAG.nonfinite(f"moe_out: {tag}", m)
        x = ops.sanitize(x + m, 1e3)
        stats.append(st)
        return x

    def forward_fused(self, x, h, next_scale, cos, sin, stats: List[Dict]):
        """Same computation with each residual update fused into the following
        RMSNorm: takes ``h = pre_norm(x)``, returns the new residual and its
        normalisation by ``next_scale`` (the next layer's ``pre_norm`` or the
        final norm)."""
        from ..ops import kernels as K
        tag = self._tag()
        delta = self.sublayer(h, cos, sin)
        DIAG.resid_breakdown(tag, x, delta)
        clip = 5e2 if self.layer_type == "mamba2" else 1e3
        # the kernel folds max |x + delta| and a non-finite-delta flag into the diagnostics
        x, h2 = K.add_rmsnorm(x, delta, self.norm_2.scale, clip, 1e-6, sanitize_delta_grad=True,
                              diag_tag=f"delta: {tag}")
        st: Dict[str, torch.Tensor] = {}
        m = self.moe(h2, st)
        stats.append(st)
        return K.add_rmsnorm(x, m, next_scale, 1e3, 1e-6, diag_tag=f"moe_out: {tag}")


class Embed(nn.Module):
    def __init__(self, vocab: int, d: int):
        super().__init__()
        # flax nn.Embed default init: variance_scaling(1, fan_in, normal, out_axis=0) -> std 1/sqrt(d)
        self.embedding = nn.Parameter(torch.randn(vocab, d) / math.sqrt(d))

    def forward(self, ids, dtype):
        if ops.use_cuda(ids):
            from ..ops import kernels as K
            return K.embedding(ids, self.embedding, dtype)
        return self.embedding.to(dtype)[ids]


class HybridMoEModel(nn.Module):
    def __init__(self, cfg: ModelConfig, compute_dtype: torch.dtype = torch.bfloat16,
                 compute_dar: bool = False, remat: bool = False):
        super().__init__()
        cfg.validate()
        self.cfg = cfg
        self.compute_dtype = compute_dtype
        self.remat = remat
        self.embed = Embed(cfg.vocab_size, cfg.d_model)
        if cfg.arch == "blockdar":
            for b in range(cfg.num_blocks):
                setattr(self, f"block_{b}", BlockDAR(cfg, b, compute_dar))
        else:
            for i in range(cfg.num_layers):
                setattr(self, f"layer_{i}", InterleavedLayer(cfg, cfg.layer_types[i]))
                getattr(self, f"layer_{i}").layer_idx = i
        self.final_norm = RMSNorm(cfg.d_model)
        if not cfg.tie_embeddings:
            self.lm_head = Dense(cfg.d_model, cfg.vocab_size)
        self._rope_cache = {}

    def has_mla(self) -> bool:
        return "mla" in self.cfg.layer_types[: self.cfg.num_layers]

    def rope(self, L: int, device):
        key = (L, str(device))
        if key not in self._rope_cache:
            self._rope_cache[key] = R.rope_cos_sin(L, self.cfg.d_head, device=device)
        return self._rope_cache[key]

    def blocks(self):
        if self.cfg.arch == "blockdar":
            return [getattr(self, f"block_{b}") for b in range(self.cfg.num_blocks)]
        return [getattr(self, f"layer_{i}") for i in range(self.cfg.num_layers)]

    def forward(self, input_ids: torch.Tensor, return_hidden: bool = True):
        """Returns ``(hidden_or_logits, stats)`` where ``stats`` is a list with one
        dict of router statistics per MoE."""
        Bsz, L = input_ids.shape
        tp = get_tp()
        if tp is not None:
            # sequence parallel: this rank embeds (and later scores) its block of the tokens
            tp.set_batch(Bsz, L)
            input_ids = tp.local_tokens(input_ids)
        cp = get_cp()
        if cp is not None:
            # context parallel: this rank holds one segment of every sequence
            cp.set_seq(L)
            input_ids = cp.local_time(input_ids)
        x = self.embed(input_ids, self.compute_dtype)
        cos, sin = self.rope(L, x.device) if self.has_mla() else (None, None)
        stats: List[Dict] = []
        if self.cfg.arch == "blockdar":
            history: List[torch.Tensor] = []
            for blk in self.blocks():
                x = blk(x, history, cos, sin, stats)
        elif self._fused_residuals(x):
            return self._forward_fused(x, cos, sin, stats, return_hidden)
        else:
            for layer in self.blocks():
                if self.remat and torch.is_grad_enabled():
                    import torch.utils.checkpoint as ckpt
                    st: List[Dict] = []
                    x = ckpt.checkpoint(layer, x, cos, sin, st, use_reentrant=False)
                    stats.extend(st)
                else:
                    with nvtx_range(f"layer/{layer.layer_type}"):
                        x = layer(x, cos, sin, stats)
        h = self.final_norm(x)
        if return_hidden:
            return h, stats
        w = self.lm_weight()
        return h @ w.to(h.dtype).t(), stats

    def _fused_residuals(self, x: torch.Tensor) -> bool:
        if not ops.use_cuda(x) or x.dtype != torch.bfloat16:
            return False
        from ..ops import kernels as K
        return K.row_fusable(self.cfg.d_model)

    def _forward_fused(self, x, cos, sin, stats: List[Dict], return_hidden: bool):
        """Interleaved stack with the residual updates fused into the RMSNorms
        that follow them (``InterleavedLayer.forward_fused``)."""
        layers = self.blocks()
        h = ops.rmsnorm(x, layers[0].pre_norm.scale, 1e-6)
        for i, layer in enumerate(layers):
            nxt = layers[i + 1].pre_norm.scale if i + 1 < len(layers) else self.final_norm.scale
            if self.remat and torch.is_grad_enabled():
                import torch.utils.checkpoint as ckpt
                st: List[Dict] = []
                x, h = ckpt.checkpoint(layer.forward_fused, x, h, nxt, cos, sin, st, use_reentrant=False)
                stats.extend(st)
            else:
                with nvtx_range(f"layer_{i}/{layer.layer_type}"):
                    x, h = layer.forward_fused(x, h, nxt, cos, sin, stats)
        if return_hidden:
            return h, stats
        return h @ self.lm_weight().to(h.dtype).t(), stats

    def token_shard(self, t: torch.Tensor) -> torch.Tensor:
        """The rows of a per-token ``(B, L, ...)`` tensor (labels) that this rank
        scores: its sequence-parallel block under tensor parallelism, else all."""
        tp = get_tp()
        if tp is not None:
            return tp.local_tokens(t)
        cp = get_cp()
        return cp.local_time(t) if cp is not None else t

    def lm_weight(self) -> torch.Tensor:
        """``(V, d)`` weight of the tied (or separate) LM head."""
        if self.cfg.tie_embeddings:
            return self.embed.embedding
        return self.lm_head.kernel.t()


def flax_path(name: str) -> str:
    """``block_0.layer_1.sublayer.gdn2.q_proj.kernel`` -> ``block_0/layer_1/...``."""
    return name.replace(".", "/")


def count_params(model: nn.Module) -> Dict[str, int]:
    tot = sum(p.numel() for p in model.parameters())
    routed = sum(p.numel() for n, p in model.named_parameters() if "routed_w" in n)
    return {"total": tot, "routed_experts": routed}


def active_params_per_token(cfg: ModelConfig, model: nn.Module) -> int:
    """Parameters touched per token (shared + top-k routed experts + LM head)."""
    tot = 0
    for n, p in model.named_parameters():
        if "routed_w" in n:
            tot += p.numel() * cfg.top_k // cfg.e_routed
        elif ".dar." in n:
            continue
        else:
            tot += p.numel()
    return tot


_ = Optional
