"""Pipeline parallelism for the interleaved stack (GPipe schedule over NCCL / gloo p2p).

The reference has no pipeline parallelism (GSPMD FSDP + DP on a 1-D mesh,
`train_setup.py:361-365`); the survey of this build lists it as optional, with the rule
that pipeline sends and receives stay on NCCL point-to-point.  Stage ``s`` of ``S`` runs a
contiguous block of the layers; the first stage also embeds the tokens and the last one
applies the final norm and the tied LM head, for which it holds a copy of the embedding
table whose gradient is summed with the first stage's before every optimizer step (both
copies then take the same update).

One optimizer step (``micro_step`` per micro-batch, then ``apply``; ``train_step`` does both): every micro-batch goes forward through
the stages (activations sent to the next stage), then every micro-batch goes backward in
the same order (activation gradients sent to the previous stage).  Each stage adds the MoE
auxiliary terms of its own layers to its backward seed, so the gradient of every
parameter is that of the single-rank loss.  The global gradient norm, the clip
coefficient and the non-finite flags are reduced over the stages.  Parameters keep their
global names, so checkpoints are interchangeable with the other layouts.
"""
from __future__ import annotations

from typing import Dict, List, Optional

import torch
import torch.distributed as dist
import torch.nn as nn


def stage_layers(num_layers: int, stages: int, stage: int) -> range:
    """Contiguous, balanced layer ranges: the first ``num_layers % stages`` stages take one more."""
    base, extra = divmod(num_layers, stages)
    lo = stage * base + min(stage, extra)
    return range(lo, lo + base + (1 if stage < extra else 0))


class PipelineStage(nn.Module):
    """The modules of one stage, registered under the model's own attribute names."""

    def __init__(self, model: nn.Module, stages: int, stage: int):
        super().__init__()
        if model.cfg.arch != "interleaved":
            raise ValueError("pipeline parallelism splits the interleaved layout")
        self.cfg = model.cfg
        self.compute_dtype = model.compute_dtype
        self.stages, self.stage = stages, stage
        self.first, self.last = stage == 0, stage == stages - 1
        self.layer_ids = list(stage_layers(model.cfg.num_layers, stages, stage))
        for i in self.layer_ids:
            setattr(self, f"layer_{i}", getattr(model, f"layer_{i}"))
        if self.first or (self.last and model.cfg.tie_embeddings):
            self.embed = model.embed
        if self.last:
            self.final_norm = model.final_norm
            if not model.cfg.tie_embeddings:
                self.lm_head = model.lm_head
        self._model = [model]  # for rope / lm_weight helpers (not a registered submodule)

    def run(self, x: torch.Tensor, seq_len: int, stats: List[Dict]) -> torch.Tensor:
        m = self._model[0]
        cos, sin = m.rope(seq_len, x.device) if m.has_mla() else (None, None)
        for i in self.layer_ids:
            x = getattr(self, f"layer_{i}")(x, cos, sin, stats)
        return x


class PipelineTrainer:
    """One pipeline stage's trainer: its own flat store and optimizer, GPipe schedule."""

    def __init__(self, model: nn.Module, stages: Optional[int] = None, total_steps: int = 1000,
                 optimizer: str = "adamw", compute_dtype: torch.dtype = torch.float32, device=None,
                 group: Optional[dist.ProcessGroup] = None, skip_nonfinite: bool = False):
        from ..optim import FlatParamStore, HybridOptimizer, grad_scale_of, label_adamw_only, label_of
        self.group = group
        self.stages = stages or dist.get_world_size(group)
        self.stage = dist.get_rank(group)
        self.ranks = [dist.get_global_rank(group, s) if group is not None else s for s in range(self.stages)]
        self.part = PipelineStage(model, self.stages, self.stage)
        self.cfg = model.cfg
        dev = device or next(model.parameters()).device
        self.device = dev
        label_fn = label_of if optimizer == "hybrid" else label_adamw_only
        tied = self.cfg.tie_embeddings and self.stages > 1 and self.part.last
        # the last stage's copy of the tied embedding sits in its own store: it takes the
        # first stage's update and is left out of the global norm
        own = (lambda n, p: not n.startswith("embed.")) if tied else None
        self.store = FlatParamStore(self.part, label_fn, grad_scale_of, 1, 0, compute_dtype=compute_dtype,
                                    device=dev, param_filter=own)
        self.opt = HybridOptimizer(self.store, total_steps, reduce_fn=self._sum_stages, skip_nonfinite=skip_nonfinite)
        self.tied_store = self.tied_opt = None
        if tied:
            self.tied_store = FlatParamStore(self.part, label_fn, grad_scale_of, 1, 0, compute_dtype=compute_dtype,
                                             device=dev, param_filter=lambda n, p: n.startswith("embed."))
            self.tied_opt = HybridOptimizer(self.tied_store, total_steps, skip_nonfinite=skip_nonfinite)
            self.tied_opt.schedule = self.opt.schedule
            self.tied_opt.norm_share = 0.0
            self.opt.partners.append(self.tied_opt)
        # first and last stage share the embedding gradient
        self.tied_group = None
        if self.cfg.tie_embeddings and self.stages > 1:
            self.tied_group = dist.new_group([self.ranks[0], self.ranks[-1]])
        n_moe = len(self.part.layer_ids)
        self._frac = torch.zeros(max(n_moe, 1), self.cfg.e_routed, device=dev)
        self.global_step = 0
        self._keep: List = []
        self._loss_sum = torch.zeros((), device=dev)

    # ------------------------------------------------------------ plumbing
    def _sum_stages(self, t: torch.Tensor) -> torch.Tensor:
        dist.all_reduce(t, group=self.group)
        return t

    def _send(self, t: torch.Tensor, stage: int) -> None:
        dist.send(t.detach().contiguous(), self.ranks[stage], group=self.group)

    def _recv(self, like_shape, dtype, stage: int) -> torch.Tensor:
        t = torch.empty(like_shape, dtype=dtype, device=self.device)
        dist.recv(t, self.ranks[stage], group=self.group)
        return t

    def _aux(self, stats: List[Dict]) -> torch.Tensor:
        from ..training.loss import ROUTER_COLLINEARITY_COEF
        zero = torch.zeros((), device=self.device)
        if not stats:
            return zero
        aux = sum(s["aux_loss"] for s in stats)
        z = sum(s["z_loss"] for s in stats)
        coll = sum(s["router_collinearity"] for s in stats)
        return self.cfg.router_aux_loss_coef * aux + self.cfg.router_z_loss_coef * z + \
            ROUTER_COLLINEARITY_COEF * coll

    # ------------------------------------------------------------ micro-step / apply (Trainer interface)
    cuda_graph = False

    @property
    def ep_store(self):  # the tied embedding copy restores / saves with the stage's stores
        return self.tied_store

    @property
    def ep_opt(self):
        return self.tied_opt

    def _forward(self, b: Dict[str, torch.Tensor], train: bool):
        """One micro-batch through this stage; returns (input, output or loss, aux, loss part)."""
        from .. import ops
        part, cfg = self.part, self.cfg
        ids = b["input_ids"]
        Bsz, L = ids.shape
        shape = (Bsz, L, cfg.d_model)
        if part.first:
            x_in = None
            x = part.embed(ids, part.compute_dtype)
        else:
            x_in = self._recv(shape, part.compute_dtype, self.stage - 1)
            if train:
                x_in.requires_grad_(True)
            x = x_in
        stats: List[Dict] = []
        x = part.run(x, L, stats)
        aux = self._aux(stats) if train else torch.zeros((), device=self.device)
        if train:
            for i, st in enumerate(stats):
                if st.get("assignment_frac") is not None:
                    self._frac[i] += st["assignment_frac"]
        part_loss = aux.detach()
        if part.last:
            h = part.final_norm(x)
            w = part.embed.embedding if cfg.tie_embeddings else part.lm_head.kernel.t()
            s, cnt = ops.cross_entropy(h, b["labels"], w, cfg.label_smoothing)
            ce = s / cnt.clamp_min(1.0)
            return x_in, ce + aux, None, part_loss + ce.detach()
        self._send(x, self.stage + 1)
        return x_in, x, aux, part_loss

    def micro_step(self, batch: Dict[str, torch.Tensor]):
        """Forward of one micro-batch on this stage (the backward runs in ``apply``)."""
        if not self._keep:
            self._frac.zero_()
        self.part.train()
        x_in, out, aux, part_loss = self._forward(batch, True)
        self._keep.append((x_in, out, aux))
        self._loss_sum += part_loss
        return part_loss, {}

    def apply(self, n_accum: Optional[int] = None) -> Dict[str, torch.Tensor]:
        """Backward of every kept micro-batch (same order as the forwards), the tied
        embedding gradient sum, then the optimizer step on this stage's parameters."""
        n = n_accum if n_accum is not None else max(len(self._keep), 1)
        for x_in, out, aux in self._keep:
            if self.part.last:
                out.backward()
            else:
                g = self._recv(out.shape, out.dtype, self.stage + 1)
                torch.autograd.backward([out, aux], [g, torch.ones_like(aux)])
            if x_in is not None:
                self._send(x_in.grad, self.stage - 1)
        if self.tied_group is not None and (self.part.first or self.part.last):
            st = self.tied_store if self.part.last else self.store
            dist.all_reduce(st.grad_view(st.by_name["embed.embedding"]), group=self.tied_group)
        out = self.opt.step(n, self._frac / max(len(self._keep), 1))
        loss = self._loss_sum.clone()
        dist.all_reduce(loss, group=self.group)  # the single-rank loss: CE + every layer's terms
        out["loss"] = loss / max(len(self._keep), 1)
        self.reset_accumulators()
        self.global_step += 1
        return out

    def reset_accumulators(self) -> None:
        self._keep = []
        self._loss_sum = torch.zeros((), device=self.device)
        self.store.zero_grad()
        if self.tied_store is not None:
            self.tied_store.zero_grad()

    def train_step(self, micro_batches: List[Dict[str, torch.Tensor]]) -> Dict[str, torch.Tensor]:
        for b in micro_batches:
            self.micro_step(b)
        return self.apply(len(micro_batches))

    @torch.no_grad()
    def eval_loss(self, batch: Dict[str, torch.Tensor]) -> torch.Tensor:
        self.part.eval()
        _, out, _, _ = self._forward(batch, False)
        loss = out.detach().reshape(()) if self.part.last else torch.zeros((), device=self.device)
        dist.all_reduce(loss, group=self.group)
        self.part.train()
        return loss

    def close(self) -> None:
        pass
