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
from ..parallel.cp import get_cp
from ..parallel.tp import get_tp, mark_shard, shard_tensor, tp_rmsnorm
from ..utils.diag import DIAG
from .layers import Dense, RMSNorm, lecun_normal_, tp_world_rank


def _shard_vec(full: torch.Tensor) -> nn.Parameter:
    """A per-channel / per-head parameter from its full-size initial value: under tensor
    parallelism this rank's piece of it (every rank draws the full value)."""
    W, rank = tp_world_rank()
    if W <= 1:
        return nn.Parameter(full)
    p = nn.Parameter(shard_tensor(full, 0, 1, W, rank).clone())
    mark_shard(p, 0)
    return p


def _conv_param(d: int, width: int, std: float = 0.02) -> nn.Parameter:
    return _shard_vec(torch.randn(d, width) * std)


class GatedDeltaNet2(nn.Module):
    """GDN-2 sublayer with per-channel decay ``g``, erase ``b`` and write ``w`` gates.

    With tensor parallelism each rank holds ``n_heads / W`` heads: the seven input
    projections are column-parallel over the gathered token rows, the conv, gates and
    scan are per channel / head, ``out_norm`` normalises over all heads (all-reduced
    statistics) and ``out_proj`` is row-parallel."""

    def __init__(self, cfg: ModelConfig):
        super().__init__()
        d = cfg.d_model
        W, _ = tp_world_rank()
        if cfg.n_heads % W:
            raise ValueError(f"{cfg.n_heads} GDN heads do not split over {W} tensor-parallel ranks")
        self.cfg = cfg
        self.tp_world = W
        self.n_heads = cfg.n_heads // W
        self.d_head = d // cfg.n_heads
        dl = d // W
        self.q_proj = Dense(d, d, tp="col")
        self.k_proj = Dense(d, d, tp="col")
        self.v_proj = Dense(d, d, tp="col")
        for n in ("q", "k", "v"):
            setattr(self, f"{n}_conv_w", _conv_param(d, cfg.d_conv))
            setattr(self, f"{n}_conv_b", _shard_vec(torch.zeros(d)))
        self.erase_gate = Dense(d, d, bias=True, tp="col")
        self.write_gate = Dense(d, d, bias=True, tp="col")
        self.decay_a = _shard_vec(torch.zeros(cfg.n_heads))
        self.decay_proj = Dense(d, d, bias=True, tp="col")
        self.out_gate = Dense(d, d, tp="col")
        self.out_norm = RMSNorm(d, tp=True)
        self.out_proj = Dense(d, d, tp="row")

    def projections(self, x: torch.Tensor):
        """``(q, k, v, erase, write, decay, out_gate)`` pre-activations over full
        sequences ``(B, L, d / W)`` (the token rows gathered under tensor parallelism)."""
        mods = (self.q_proj, self.k_proj, self.v_proj, self.erase_gate, self.write_gate, self.decay_proj,
                self.out_gate)
        tp = get_tp()
        if tp is not None:
            return tp.gather_linear(x, [(m.kernel, m.bias) for m in mods])
        if ops.use_cuda(x) and x.dtype == torch.bfloat16:
            from ..ops import kernels as K
            return list(K.linear_multi(x, [(m.kernel, m.bias) for m in mods]))
        return [m(x) for m in mods]

    def out_projection(self, o: torch.Tensor) -> torch.Tensor:
        tp = get_tp()
        if tp is not None:
            return tp.linear_scatter(o, self.out_proj.kernel)
        return self.out_proj(o)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        cp = get_cp()
        if ops.use_cuda(x) and cp is None:
            return self._forward_fused(x)
        H, D = self.n_heads, self.d_head
        qp, kp, vp, bp, wp, fp, og = self.projections(x)
        Bsz, L, dl = qp.shape
        conv = ops.conv1d if cp is None else (lambda t, w_, b_, **kw: cp.causal_conv(ops.conv1d, t, w_, b_, **kw))
        q = conv(qp, self.q_conv_w, self.q_conv_b, silu=True)
        k = conv(kp, self.k_conv_w, self.k_conv_b, silu=True)
        v = conv(vp, self.v_conv_w, self.v_conv_b, silu=True, clip=50.0)
        q = q.view(Bsz, L, H, D)
        k = k.view(Bsz, L, H, D)
        v = v.view(Bsz, L, H, D)
        q = ops.grad_sanitize(R.safe_l2norm(q, 1e-12))
        k = ops.grad_sanitize(R.safe_l2norm(k, 1e-12))
        b_gate = torch.sigmoid(bp).view(Bsz, L, H, D)
        w_gate = torch.sigmoid(wp).view(Bsz, L, H, D)
        f = fp.view(Bsz, L, H, D).float()
        g = -torch.exp(self.decay_a.float().clamp(-20.0, 20.0))[None, None, :, None] * F.softplus(f)
        g = torch.nan_to_num(g, nan=0.0, posinf=0.0, neginf=-20.0)
        og = og.clamp(-1e2, 1e2)
        q, k, v, w_gate, b_gate = (R.sanitize(t, 1e3) for t in (q, k, v, w_gate, b_gate))
        g = R.sanitize(g, 1e3)
        for name, t in (("q", q), ("k", k), ("v", v), ("g", g)):
            DIAG.stage("GDN2", name, t)
        if cp is not None:
            o = cp.gdn2_scan(q, k, v, g, b_gate, w_gate, 1.0, self.cfg.gdn_chunk).reshape(Bsz, L, dl)
        else:
            o = ops.gdn2(q, k, v, w_gate, b_gate, g, 1.0, self.cfg.gdn_chunk).reshape(Bsz, L, dl)
        DIAG.stage("GDN2", "o", o)
        tp = get_tp()
        if tp is not None:
            o = tp_rmsnorm(o, self.out_norm.scale, 1e-6, self.cfg.d_model, tp).to(o.dtype)
        else:
            o = self.out_norm(o)
        return self.out_projection(o * F.silu(og))

    def _forward_fused(self, x: torch.Tensor) -> torch.Tensor:
        from ..ops import kernels as K
        return K.gdn2_layer(self, x)


class Mamba2(nn.Module):
    """Mamba2 sublayer: per-head ``A``, per-channel ``dt``, B/C shared by all heads.

    With tensor parallelism each rank holds ``n_heads_ssm / W`` heads: ``in_proj``
    is column-parallel (its ``x_bc`` and gate halves split alike), ``B_proj`` /
    ``C_proj`` (replicated) and ``dt_proj`` (column-parallel) read the full ``x_bc``
    gathered along features, and ``out_proj`` is row-parallel."""

    def __init__(self, cfg: ModelConfig):
        super().__init__()
        d, di, N = cfg.d_model, cfg.d_inner, cfg.d_state
        W, rank = tp_world_rank()
        if cfg.n_heads_ssm % W:
            raise ValueError(f"{cfg.n_heads_ssm} SSM heads do not split over {W} tensor-parallel ranks")
        self.cfg = cfg
        self.tp_world = W
        dil = di // W
        self.n_heads = cfg.n_heads_ssm // W
        self.in_proj = Dense(d, 2 * di, tp="col2")
        self.conv_w = _conv_param(di, cfg.d_conv)
        self.conv_b = _shard_vec(torch.zeros(di))
        if cfg.ssm_init == "mamba":
            a_log = torch.empty(cfg.n_heads_ssm).uniform_(0.0, math.log(16.0))
        else:
            a_log = torch.rand(cfg.n_heads_ssm)
        self.A_log = _shard_vec(a_log)
        self.B_proj = Dense(di, N)
        self.C_proj = Dense(di, N)
        self.dt_proj = Dense(di, di, bias=True, tp="col")
        if cfg.ssm_init == "mamba":
            dt0 = torch.empty(di).uniform_(1e-3, 0.1)
            dt_bias = dt0 + torch.log(-torch.expm1(-dt0))
            if W > 1:
                dt_bias = shard_tensor(dt_bias, 0, 1, W, rank)
            with torch.no_grad():
                self.dt_proj.bias.copy_(dt_bias)
        self.ssm_out_norm = RMSNorm(di, tp=True)
        self.out_proj = Dense(di, d, tp="row")

    def in_projection(self, x: torch.Tensor) -> torch.Tensor:
        tp = get_tp()
        if tp is not None:
            return tp.gather_linear(x, [(self.in_proj.kernel, None)])[0]
        return self.in_proj(x)

    def bc_input(self, x_bc: torch.Tensor) -> torch.Tensor:
        """The full ``x_bc`` (all channels) that B, C and dt are projected from."""
        tp = get_tp()
        return tp.gather_features(x_bc) if tp is not None else x_bc

    def out_projection(self, out: torch.Tensor) -> torch.Tensor:
        tp = get_tp()
        if tp is not None:
            return tp.linear_scatter(out, self.out_proj.kernel)
        return self.out_proj(out)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        cp = get_cp()
        if ops.use_cuda(x) and cp is None:
            from ..ops import kernels as K
            return K.mamba2_layer(self, x)
        Hs = self.n_heads
        xz = self.in_projection(x)
        Bsz, L, two_dil = xz.shape
        dil = two_dil // 2
        P = dil // Hs
        x_bc, res = xz[..., :dil], xz[..., dil:]
        if cp is not None:
            x_conv = cp.causal_conv(ops.conv1d, x_bc, self.conv_w, self.conv_b, silu=True)
        else:
            x_conv = ops.conv1d(x_bc, self.conv_w, self.conv_b, silu=True)
        A = -torch.exp(self.A_log.float().clamp(-20.0, 20.0))
        xin = self.bc_input(x_bc)
        Bm = self.B_proj(xin)
        Cm = self.C_proj(xin)
        dt = F.softplus(self.dt_proj(xin)).clamp(1e-2, 1.0)
        dt, Bm, Cm, x_conv = (R.sanitize(t, 1e3) for t in (dt, Bm, Cm, x_conv))
        for name, t in (("in_proj", xz), ("x_conv", x_conv), ("dt", dt)):
            DIAG.stage("MAMBA2", name, t)
        if cp is not None:
            y = cp.ssd_scan(dt.view(Bsz, L, Hs, P), A, Bm, Cm, x_conv.view(Bsz, L, Hs, P), self.cfg.ssd_chunk)
        else:
            y = ops.ssd(dt.view(Bsz, L, Hs, P), A, Bm, Cm, x_conv.view(Bsz, L, Hs, P), self.cfg.ssd_chunk)
        DIAG.stage("MAMBA2", "ssd_y", y)
        y = y.reshape(Bsz, L, dil).to(x_bc.dtype)
        tp = get_tp()
        if tp is not None:
            y = tp_rmsnorm(y, self.ssm_out_norm.scale, 1e-6, self.cfg.d_inner, tp).to(y.dtype)
        else:
            y = self.ssm_out_norm(y)
        out = (y * F.silu(res)).clamp(-3e2, 3e2)
        return self.out_projection(out)


class MLA(nn.Module):
    """Latent-KV causal attention (reference ``MLAJ``), RoPE on Q and K.

    With tensor parallelism each rank holds ``n_heads / W`` heads (``W_q``,
    ``W_k_up``, ``W_v_up`` column-parallel, ``W_o`` row-parallel); the latent
    down-projection is replicated and computed on the gathered rows."""

    def __init__(self, cfg: ModelConfig):
        super().__init__()
        d = cfg.d_model
        W, _ = tp_world_rank()
        if cfg.n_heads % W:
            raise ValueError(f"{cfg.n_heads} attention heads do not split over {W} tensor-parallel ranks")
        self.cfg = cfg
        self.tp_world = W
        self.n_heads = cfg.n_heads // W
        self.W_q = Dense(d, d, tp="col")
        self.W_kv_down = Dense(d, cfg.d_latent)
        self.W_k_up = Dense(cfg.d_latent, d, tp="col")
        self.W_v_up = Dense(cfg.d_latent, d, tp="col")
        self.attn_out_norm = RMSNorm(d, tp=True)
        self.W_o = Dense(d, d, tp="row")

    def forward(self, x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
        H = self.n_heads
        dh = self.cfg.d_model // self.cfg.n_heads
        tp = get_tp()
        if tp is not None:
            Qp, lat = tp.gather_linear(x, [(self.W_q.kernel, None), (self.W_kv_down.kernel, None)])
        else:
            Qp, lat = self.W_q(x), self.W_kv_down(x)
        Bsz, L, dl = Qp.shape
        cp = get_cp()
        q0, Lk = 0, L
        if cp is not None:  # keys / values of the whole sequence from the gathered latent
            lat = cp.gather_time(lat)
            q0, Lk = cp.seg[0], lat.shape[1]
        Q = Qp.view(Bsz, L, H, dh).transpose(1, 2)
        K = self.W_k_up(lat).view(Bsz, Lk, H, dh).transpose(1, 2)
        V = self.W_v_up(lat).view(Bsz, Lk, H, dh).transpose(1, 2)
        Q = R.apply_rope(Q, cos[q0:q0 + L, :dh], sin[q0:q0 + L, :dh])
        K = R.apply_rope(K, cos[:Lk, :dh], sin[:Lk, :dh])
        Q, K, V = (R.sanitize(t, 1e3) for t in (Q, K, V))
        if cp is not None:
            keep = torch.arange(Lk, device=Q.device)[None, :] <= (q0 + torch.arange(L, device=Q.device))[:, None]
            out = F.scaled_dot_product_attention(Q, K, V, attn_mask=keep, scale=1.0 / math.sqrt(dh))
        else:
            out = ops.attention(Q.contiguous(), K.contiguous(), V.contiguous(), 1.0 / math.sqrt(dh))
        out = out.transpose(1, 2).reshape(Bsz, L, dl)
        if tp is not None:
            out = tp_rmsnorm(out, self.attn_out_norm.scale, 1e-6, self.cfg.d_model, tp).to(out.dtype)
        else:
            out = self.attn_out_norm(out)
        out = ops.grad_sanitize(out)
        if tp is not None:
            return tp.linear_scatter(out, self.W_o.kernel)
        return self.W_o(out)


_ = lecun_normal_
