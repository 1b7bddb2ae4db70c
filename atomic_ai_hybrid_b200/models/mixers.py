"""Sequence mixers: GDN-2, Mamba2 and MLA attention.

Parameter names, shapes and the order of the clip / normalisation steps follow
the reference modules (`model.py:286-385` MLAJ, `model.py:391-525` Mamba2J,
`model.py:564-653` GatedDeltaNet2J).  The arithmetic runs through ``ops``: fused
sm_100a kernels on the GPU, plain PyTorch on the CPU or in the eager baseline.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from .. import ops
from ..config import ModelConfig
from ..ops import reference as R
from .layers import Dense, RMSNorm, lecun_normal_


def _conv_param(d: int, width: int, std: float = 0.02) -> nn.Parameter:
    return nn.Parameter(torch.randn(d, width) * std)


class GatedDeltaNet2(nn.Module):
    """GDN-2 sublayer with per-channel decay ``g``, erase ``b`` and write ``w`` gates."""

    def __init__(self, cfg: ModelConfig):
        super().__init__()
        d = cfg.d_model
        self.cfg = cfg
        self.n_heads = cfg.n_heads
        self.d_head = d // cfg.n_heads
        self.q_proj = Dense(d, d)
        self.k_proj = Dense(d, d)
        self.v_proj = Dense(d, d)
        for n in ("q", "k", "v"):
            setattr(self, f"{n}_conv_w", _conv_param(d, cfg.d_conv))
            setattr(self, f"{n}_conv_b", nn.Parameter(torch.zeros(d)))
        self.erase_gate = Dense(d, d, bias=True)
        self.write_gate = Dense(d, d, bias=True)
        self.decay_a = nn.Parameter(torch.zeros(cfg.n_heads))
        self.decay_proj = Dense(d, d, bias=True)
        self.out_gate = Dense(d, d)
        self.out_norm = RMSNorm(d)
        self.out_proj = Dense(d, d)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        Bsz, L, d = x.shape
        H, D = self.n_heads, self.d_head
        if ops.use_cuda(x):
            return self._forward_fused(x)
        q = ops.conv1d(self.q_proj(x), self.q_conv_w, self.q_conv_b, silu=True)
        k = ops.conv1d(self.k_proj(x), self.k_conv_w, self.k_conv_b, silu=True)
        v = ops.conv1d(self.v_proj(x), self.v_conv_w, self.v_conv_b, silu=True, clip=50.0)
        q = q.view(Bsz, L, H, D)
        k = k.view(Bsz, L, H, D)
        v = v.view(Bsz, L, H, D)
        q = ops.grad_sanitize(R.safe_l2norm(q, 1e-12))
        k = ops.grad_sanitize(R.safe_l2norm(k, 1e-12))
        b_gate = torch.sigmoid(self.erase_gate(x)).view(Bsz, L, H, D)
        w_gate = torch.sigmoid(self.write_gate(x)).view(Bsz, L, H, D)
        f = self.decay_proj(x).view(Bsz, L, H, D).float()
        g = -torch.exp(self.decay_a.float().clamp(-20.0, 20.0))[None, None, :, None] * F.softplus(f)
        g = torch.nan_to_num(g, nan=0.0, posinf=0.0, neginf=-20.0)
        og = self.out_gate(x).clamp(-1e2, 1e2)
        q, k, v, w_gate, b_gate = (R.sanitize(t, 1e3) for t in (q, k, v, w_gate, b_gate))
        g = R.sanitize(g, 1e3)
        o = ops.gdn2(q, k, v, w_gate, b_gate, g, 1.0, self.cfg.gdn_chunk).reshape(Bsz, L, d)
        o = self.out_norm(o)
        return self.out_proj(o * F.silu(og))

    def _forward_fused(self, x: torch.Tensor) -> torch.Tensor:
        from ..ops import kernels as K
        return K.gdn2_layer(self, x)


class Mamba2(nn.Module):
    """Mamba2 sublayer: per-head ``A``, per-channel ``dt``, B/C shared by all heads."""

    def __init__(self, cfg: ModelConfig):
        super().__init__()
        d, di, N = cfg.d_model, cfg.d_inner, cfg.d_state
        self.cfg = cfg
        self.in_proj = Dense(d, 2 * di)
        self.conv_w = _conv_param(di, cfg.d_conv)
        self.conv_b = nn.Parameter(torch.zeros(di))
        if cfg.ssm_init == "mamba":
            a_log = torch.empty(cfg.n_heads_ssm).uniform_(0.0, math.log(16.0))
        else:
            a_log = torch.rand(cfg.n_heads_ssm)
        self.A_log = nn.Parameter(a_log)
        self.B_proj = Dense(di, N)
        self.C_proj = Dense(di, N)
        self.dt_proj = Dense(di, di, bias=True)
        if cfg.ssm_init == "mamba":
            dt0 = torch.empty(di).uniform_(1e-3, 0.1)
            with torch.no_grad():
                self.dt_proj.bias.copy_(dt0 + torch.log(-torch.expm1(-dt0)))
        self.ssm_out_norm = RMSNorm(di)
        self.out_proj = Dense(di, d)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if ops.use_cuda(x):
            from ..ops import kernels as K
            return K.mamba2_layer(self, x)
        Bsz, L, d = x.shape
        di, Hs = self.cfg.d_inner, self.cfg.n_heads_ssm
        P = di // Hs
        xz = self.in_proj(x)
        x_bc, res = xz[..., :di], xz[..., di:]
        x_conv = ops.conv1d(x_bc, self.conv_w, self.conv_b, silu=True)
        A = -torch.exp(self.A_log.float().clamp(-20.0, 20.0))
        Bm = self.B_proj(x_bc)
        Cm = self.C_proj(x_bc)
        dt = F.softplus(self.dt_proj(x_bc)).clamp(1e-2, 1.0)
        dt, Bm, Cm, x_conv = (R.sanitize(t, 1e3) for t in (dt, Bm, Cm, x_conv))
        y = ops.ssd(dt.view(Bsz, L, Hs, P), A, Bm, Cm, x_conv.view(Bsz, L, Hs, P), self.cfg.ssd_chunk)
        y = self.ssm_out_norm(y.reshape(Bsz, L, di).to(x_bc.dtype))
        out = (y * F.silu(res)).clamp(-3e2, 3e2)
        return self.out_proj(out)


class MLA(nn.Module):
    """Latent-KV causal attention (reference ``MLAJ``), RoPE on Q and K."""

    def __init__(self, cfg: ModelConfig):
        super().__init__()
        d = cfg.d_model
        self.cfg = cfg
        self.W_q = Dense(d, d)
        self.W_kv_down = Dense(d, cfg.d_latent)
        self.W_k_up = Dense(cfg.d_latent, d)
        self.W_v_up = Dense(cfg.d_latent, d)
        self.attn_out_norm = RMSNorm(d)
        self.W_o = Dense(d, d)

    def forward(self, x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
        Bsz, L, d = x.shape
        H = self.cfg.n_heads
        dh = d // H
        Q = self.W_q(x).view(Bsz, L, H, dh).transpose(1, 2)
        lat = self.W_kv_down(x)
        K = self.W_k_up(lat).view(Bsz, L, H, dh).transpose(1, 2)
        V = self.W_v_up(lat).view(Bsz, L, H, dh).transpose(1, 2)
        Q = R.apply_rope(Q, cos[:L, :dh], sin[:L, :dh])
        K = R.apply_rope(K, cos[:L, :dh], sin[:L, :dh])
        Q, K, V = (R.sanitize(t, 1e3) for t in (Q, K, V))
        out = ops.attention(Q.contiguous(), K.contiguous(), V.contiguous(), 1.0 / math.sqrt(dh))
        out = out.transpose(1, 2).reshape(Bsz, L, d)
        out = self.attn_out_norm(out)
        out = ops.grad_sanitize(out)
        return self.W_o(out)


_ = lecun_normal_
