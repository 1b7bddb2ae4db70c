"""Dropless top-k MoE with a shared expert (reference ``GmmMoEJ``,
`atomic_ops/moe_gmm.py:342-602`).

Router (reference `atomic_ops/moe_gmm.py:409-507`):

* the router kernel ``(d, E)`` is used with L2-normalised columns, the input
  rows are L2-normalised, and the cosine logits are scaled by a learned
  temperature ``router_temp`` clipped to ``[1, 15]``;
* logits are clipped to ``+-8``; Gaussian noise is added in training;
* ``expert_bias`` (no gradient) is added only for the top-k *selection*; the
  gate is the softmax over the unbiased logits of the selected experts;
* statistics: aux (``E * sum(mean_probs^2)`` over the full softmax), z
  (``mean(logsumexp^2)``), router collinearity (mean squared off-diagonal of the
  column Gram matrix), max |cos|, input-norm stats and assignment fractions.

Dispatch is dropless: the ``k`` copies of every token are grouped by expert and
run through the grouped FFN (GELU or SwiGLU), then combined with the gates.
"""
from __future__ import annotations

from typing import Dict

import torch
import torch.nn as nn
import torch.nn.functional as F

from .. import ops
from ..config import ModelConfig
from ..ops import reference as R
from ..parallel.context import dp_mean, get_parallel_context
from .layers import Dense, lecun_normal_

ROUTER_LOGIT_CLIP = 8.0
ROUTER_TEMP_INIT = 10.0


class MoE(nn.Module):
    def __init__(self, cfg: ModelConfig):
        super().__init__()
        d, F_ = cfg.d_model, cfg.d_ff
        E = cfg.e_routed
        self.cfg = cfg
        self.E = E
        self.k = cfg.top_k
        self.swiglu = cfg.ffn_act == "swiglu"
        self.n_shared = cfg.n_shared_experts
        if self.n_shared > 0:
            Fs = F_ * self.n_shared
            self.shared_w1 = Dense(d, Fs, bias=True)
            if self.swiglu:
                self.shared_w3 = Dense(d, Fs, bias=True)
            self.shared_w2 = Dense(Fs, d, bias=True)
        self.router = nn.Parameter(torch.empty(d, E))
        lecun_normal_(self.router.data, d)
        self.router_temp = nn.Parameter(torch.tensor(ROUTER_TEMP_INIT))
        self.expert_bias = nn.Parameter(torch.zeros(E), requires_grad=False)
        # Routed expert weights are bf16 in the reference's parameter tree.  With expert
        # parallelism this rank holds experts [ep_rank * El, (ep_rank + 1) * El) only.
        pc = get_parallel_context()
        self.ep_world, self.ep_rank = pc.ep_world, pc.ep_rank
        if E % self.ep_world:
            raise ValueError(f"{E} routed experts do not split over {self.ep_world} expert-parallel ranks")
        El = E // self.ep_world
        lo = self.ep_rank * El

        def experts(rows: int, cols: int) -> nn.Parameter:
            # every rank draws all E experts (same seed, same order) and keeps its block, so the
            # initial model does not depend on the expert-parallel layout
            full = lecun_normal_(torch.empty(E, rows, cols), rows)
            return nn.Parameter(full[lo:lo + El].clone() if self.ep_world > 1 else full)

        self.routed_w1 = experts(d, F_)
        self.routed_w2 = experts(F_, d)
        self.routed_w3 = experts(d, F_) if self.swiglu else None
        if self.ep_world > 1:
            for w in (self.routed_w1, self.routed_w2, self.routed_w3):
                if w is not None:
                    w._ahb_ep_local = True

    # ------------------------------------------------------------------ router
    def route(self, flat_x: torch.Tensor, stats: Dict[str, torch.Tensor]):
        E, k = self.E, self.k
        if ops.use_cuda(flat_x) and flat_x.dtype == torch.bfloat16:
            from ..ops import kernels as K
            if K.router_supported(flat_x.shape[1], E, k):
                return self._route_fused(flat_x, stats)
        xr = ops.grad_sanitize(flat_x).float()
        nrm = xr.norm(dim=1)
        stats["norm_x_mean"] = nrm.mean().detach()
        stats["norm_x_max"] = nrm.max().detach()
        stats["norm_x_min"] = nrm.min().detach()
        kern = self.router.float()
        kn = kern * torch.rsqrt((kern * kern).sum(0, keepdim=True) + 1e-6)
        gram = kn.t() @ kn
        eye = torch.eye(E, device=gram.device, dtype=gram.dtype)
        stats["router_collinearity"] = ((gram - eye).square() * (1 - eye)).sum() / (E * (E - 1))
        stats["router_max_cos"] = (gram - eye).abs().max().detach()
        temp = self.router_temp.float().clamp(1.0, 15.0)
        xn = xr * torch.rsqrt((xr * xr).sum(-1, keepdim=True) + 1e-6)
        logits = (xn @ kn) * temp
        stats["max_abs_logit_preclip"] = logits.abs().max().detach()
        stats["min_col_norm"] = kern.square().sum(0).sqrt().min().detach()
        logits = R.sanitize(logits.clamp(-ROUTER_LOGIT_CLIP, ROUTER_LOGIT_CLIP), 1e3)
        if self.training and self.cfg.router_noise_std > 0:
            logits = logits + self.cfg.router_noise_std * torch.randn_like(logits)
        biased = logits + self.expert_bias.detach().float()[None, :]
        top_idx = torch.topk(biased, k, dim=-1).indices
        gate = torch.softmax(logits.gather(1, top_idx), dim=-1)
        counts = torch.zeros(E, device=flat_x.device, dtype=torch.float32).scatter_add_(
            0, top_idx.reshape(-1), torch.ones(top_idx.numel(), device=flat_x.device, dtype=torch.float32))
        stats["assignment_frac"] = (counts / (flat_x.shape[0] * k)).detach()
        probs = torch.nan_to_num(torch.softmax(logits, -1), nan=0.0, posinf=0.0, neginf=0.0)
        mean_probs = dp_mean(probs.mean(0))  # batch-global, as the reference's GSPMD mean
        stats["aux_loss"] = E * (mean_probs * mean_probs).sum()
        stats["z_loss"] = torch.logsumexp(logits, -1).square().mean()
        stats["expert_utilization"] = mean_probs.detach()
        stats["router_temp"] = self.router_temp.detach().float()
        stats["expert_bias"] = self.expert_bias.detach().float()
        stats["moe_dropped_ratio"] = torch.zeros((), device=flat_x.device)
        return top_idx, gate

    def _route_fused(self, flat_x: torch.Tensor, stats: Dict[str, torch.Tensor]):
        """Same router with the (T, d) work in one sm_100a kernel (``ops.kernels.router``):
        the (d, E) column normalisation, Gram statistics and loss reductions stay here."""
        from ..ops import kernels as K
        E, k = self.E, self.k
        T = flat_x.shape[0]
        kern = self.router.float()
        kn = kern * torch.rsqrt((kern * kern).sum(0, keepdim=True) + 1e-6)
        gram = kn.t() @ kn
        eye = torch.eye(E, device=gram.device, dtype=gram.dtype)
        stats["router_collinearity"] = ((gram - eye).square() * (1 - eye)).sum() / (E * (E - 1))
        stats["router_max_cos"] = (gram - eye).abs().max().detach()
        temp = self.router_temp.float().clamp(1.0, 15.0).reshape(1)
        noise = None
        if self.training and self.cfg.router_noise_std > 0:
            noise = self.cfg.router_noise_std * torch.randn(T, E, device=flat_x.device)
        gate, psum, lse_sq, top_idx, counts, scal = K.router(flat_x, kn, temp, self.expert_bias.detach().float(),
                                                             noise, k)
        stats["norm_x_mean"] = (scal[2] / T).detach()
        stats["norm_x_max"] = scal[3].detach()
        stats["norm_x_min"] = scal[4].detach()
        stats["max_abs_logit_preclip"] = scal[1].detach()
        stats["min_col_norm"] = kern.square().sum(0).sqrt().min().detach()
        stats["assignment_frac"] = (counts / (T * k)).detach()
        mean_probs = dp_mean(psum / T)  # batch-global, as the reference's GSPMD mean
        stats["aux_loss"] = E * (mean_probs * mean_probs).sum()
        stats["z_loss"] = lse_sq.reshape(()) / T
        stats["expert_utilization"] = mean_probs.detach()
        stats["router_temp"] = self.router_temp.detach().float()
        stats["expert_bias"] = self.expert_bias.detach().float()
        stats["moe_dropped_ratio"] = torch.zeros((), device=flat_x.device)
        return top_idx, gate

    # ------------------------------------------------------------------ forward
    def _shared(self, flat: torch.Tensor) -> torch.Tensor:
        if self.swiglu:
            if ops.use_cuda(flat) and flat.dtype == torch.bfloat16:
                from ..ops import kernels as K
                h1, h3 = K.linear_multi(flat, [(self.shared_w1.kernel, self.shared_w1.bias),
                                               (self.shared_w3.kernel, self.shared_w3.bias)])
                h = K.swiglu(h1, h3)
            else:
                h1, h3 = self.shared_w1(flat), self.shared_w3(flat)
                h = F.silu(h1) * h3
        else:
            h = R.gelu_tanh(self.shared_w1(flat))
        if self.training and self.cfg.dropout_rate > 0:
            h = F.dropout(h, self.cfg.dropout_rate)
        return self.shared_w2(h)

    def forward(self, x: torch.Tensor, stats: Dict[str, torch.Tensor]) -> torch.Tensor:
        Bsz, L, d = x.shape
        flat = x.reshape(-1, d)
        top_idx, gate = self.route(flat, stats)
        shared = self._shared(flat) if self.n_shared > 0 else None
        if self.ep_world > 1:
            pc = get_parallel_context()
            act = "swiglu" if self.swiglu else "gelu"
            if pc.ep is not None and ops.use_cuda(flat):
                from ..parallel.ep import moe_forward_ep
                out = moe_forward_ep(flat, top_idx, gate, self.routed_w1, self.routed_w2, self.routed_w3, shared,
                                     act, pc.ep)
                return out.view(Bsz, L, d)
            # no peer buffers (CPU, or the NCCL baseline): all-to-all through torch.distributed
            from ..parallel.ep import moe_forward_ep_collective
            out = moe_forward_ep_collective(flat, top_idx, gate, self.routed_w1, self.routed_w2, self.routed_w3,
                                            act, pc.ep_group, self.ep_world, self.ep_rank, self.E)
            if shared is not None:
                out = out + shared.float()
            return R.sanitize(out, 1e3).view(Bsz, L, d).to(x.dtype)
        # the grouped GEMM tiles need d_model and d_ff in multiples of 256
        if ops.use_cuda(flat) and x.dtype == torch.bfloat16 and d % 256 == 0 and self.cfg.d_ff % 256 == 0:
            from ..ops import kernels as K
            out = K.moe_forward(flat, top_idx, gate, self.routed_w1, self.routed_w2, self.routed_w3, shared,
                                "swiglu" if self.swiglu else "gelu")
            return out.view(Bsz, L, d)
        out = self._routed_eager(flat, top_idx, gate)
        if shared is not None:
            out = out + shared.float()
        out = R.sanitize(out.float(), 1e3)
        return out.view(Bsz, L, d).to(x.dtype)

    def _routed_eager(self, flat, top_idx, gate):
        T, d = flat.shape
        k = self.k
        # k copies ordered [all tokens for choice 0][all tokens for choice 1]...
        eidx = top_idx.t().reshape(-1)
        perm = torch.argsort(eidx, stable=True)
        sizes = torch.bincount(eidx, minlength=self.E)
        rows = perm % T
        xs = flat[rows]
        y = ops.grouped_ffn(xs, sizes, self.routed_w1, self.routed_w2, self.routed_w3,
                            "swiglu" if self.swiglu else "gelu", group_sizes_cpu=sizes.tolist())
        y = R.sanitize(y.float(), 1e3)
        w = gate.t().reshape(-1)[perm]
        out = torch.zeros(T, d, device=flat.device, dtype=torch.float32)
        out.index_add_(0, rows, y * w[:, None])
        return out
