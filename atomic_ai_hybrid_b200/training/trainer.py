"""Train step: gradient accumulation over micro-batches, then the sharded apply.

One ``Trainer`` per process (one process per GPU).  ``micro_step`` runs the
forward/backward of one micro-batch and accumulates fp32 gradients in the flat
store (reference ``distributed_train_step_micro``, `train_setup.py:477-488`);
``apply`` reduces gradients across the data-parallel group onto their owner
ranks, runs the hybrid optimizer on the owned shard and gathers the updated
weights back to every rank (reference ``distributed_apply_step``,
`train_setup.py:490-550`).  The assignment fractions used by the expert-bias
hook are averaged over the micro-steps of the step and over ranks.
"""
from __future__ import annotations

from typing import Dict, List, Optional

import torch
import torch.distributed as dist

from ..optim import FlatParamStore, HybridOptimizer, grad_scale_of, label_adamw_only, label_of
from .loss import compute_loss


class Trainer:
    def __init__(self, model, total_steps: int = 1000, optimizer: str = "hybrid",
                 compute_dtype: torch.dtype = torch.bfloat16, device=None,
                 group: Optional[dist.ProcessGroup] = None, comm: str = "auto",
                 ce_chunk_size: int = 2048, collinearity_coef: Optional[float] = None,
                 skip_nonfinite: bool = False):
        self.model = model
        self.cfg = model.cfg
        self.group = group
        dist_on = dist.is_available() and dist.is_initialized()
        self.world = dist.get_world_size(group) if dist_on else 1
        self.rank = dist.get_rank(group) if dist_on else 0
        label_fn = label_of if optimizer == "hybrid" else label_adamw_only
        self.store = FlatParamStore(model, label_fn, grad_scale_of, self.world, self.rank,
                                    compute_dtype=compute_dtype, device=device)
        self.comm = None
        if self.world > 1:
            from ..parallel.fsdp import make_shard_comm
            self.comm = make_shard_comm(self.store, group, comm)
        self.opt = HybridOptimizer(self.store, total_steps, reduce_fn=self._allreduce_sum,
                                   skip_nonfinite=skip_nonfinite)
        self.ce_chunk_size = ce_chunk_size
        self.collinearity_coef = collinearity_coef
        self._frac: List[torch.Tensor] = []
        self.global_step = 0

    def _allreduce_sum(self, t: torch.Tensor) -> torch.Tensor:
        if self.world > 1:
            dist.all_reduce(t, group=self.group)
        return t

    def micro_step(self, batch: Dict[str, torch.Tensor]):
        self.model.train()
        loss, info = compute_loss(self.model, batch, deterministic=False, ce_chunk_size=self.ce_chunk_size,
                                  collinearity_coef=self.collinearity_coef)
        loss.backward()
        if info.get("assignment_frac") is not None:
            self._frac.append(info["assignment_frac"])
        return loss.detach(), info

    def apply(self, n_accum: int) -> Dict[str, torch.Tensor]:
        frac = None
        if self._frac:
            frac = torch.stack(self._frac).mean(0)
            if self.world > 1:
                dist.all_reduce(frac, group=self.group)
                frac = frac / self.world
        self._frac = []
        if self.comm is not None:
            self.comm.reduce_scatter_grads()
        out = self.opt.step(n_accum, frac)
        if self.comm is not None:
            self.comm.all_gather_params()
        self.store.zero_grad()
        self.global_step += 1
        return out

    def train_step(self, micro_batches: List[Dict[str, torch.Tensor]]):
        losses = []
        for b in micro_batches:
            loss, _ = self.micro_step(b)
            losses.append(loss)
        out = self.apply(len(micro_batches))
        out["loss"] = torch.stack(losses).mean()
        return out

    @torch.no_grad()
    def eval_loss(self, batch: Dict[str, torch.Tensor]) -> torch.Tensor:
        self.model.eval()
        loss, _ = compute_loss(self.model, batch, deterministic=True, ce_chunk_size=self.ce_chunk_size)
        self.model.train()
        return loss
