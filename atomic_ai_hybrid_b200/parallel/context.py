"""Process-group context shared by the model and the trainer.

The reference runs on a 1-D device mesh (``("tpu_nodes",)``, reference
`train_setup.py:361-365`, ``set_model_mesh``/``get_model_mesh`` in
`model.py:81-93`).  Here one process drives one GPU and the groups are explicit:

* ``dp``: the ranks that hold different tokens (data parallel, and with sequence
  parallelism the tensor-parallel ranks too); batch-global statistics average over it,
* ``ep``: expert parallel (routed experts split across ranks),
* ``tp``: tensor parallel (heads split across ranks, token rows split between the
  mixers; ``parallel.tp``).

Batch-global statistics that the reference computes over the whole sharded
batch (the MoE load-balancing mean probabilities) are averaged over ``dp`` with a
differentiable all-reduce, so data-parallel training matches single-device
training on the global batch.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist


@dataclass
class ParallelContext:
    dp_group: Optional[dist.ProcessGroup] = None
    dp_world: int = 1
    ep_group: Optional[dist.ProcessGroup] = None
    ep_world: int = 1
    tp_group: Optional[dist.ProcessGroup] = None
    tp_world: int = 1
    ep_rank: int = 0
    ep: Optional[object] = None  # the EPGroup (peer buffers) once built
    tp_rank: int = 0
    tp: Optional[object] = None  # the TPGroup (token layout, collectives)
    cp: Optional[object] = None  # the CPGroup (sequence segments; parallel.cp)
    # ranks that hold the same rank-local parameters (data-parallel replicas of a
    # tensor- or expert-parallel group); None when every such piece has one owner
    local_group: Optional[dist.ProcessGroup] = None


_CTX = ParallelContext()


def set_parallel_context(ctx: ParallelContext) -> None:
    global _CTX
    _CTX = ctx


def get_parallel_context() -> ParallelContext:
    return _CTX


def dp_mean(t: torch.Tensor) -> torch.Tensor:
    """Differentiable mean over the data-parallel group (identity when dp == 1)."""
    ctx = _CTX
    if ctx.dp_world <= 1 or not dist.is_initialized():
        return t
    import torch.distributed.nn.functional as dfn
    return dfn.all_reduce(t, op=dist.ReduceOp.SUM, group=ctx.dp_group) / ctx.dp_world
