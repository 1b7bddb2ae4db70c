"""Basic parameter-holding layers with the reference's flax parameter names.

Every ``Dense`` stores ``kernel`` with the flax layout ``(in, out)`` and an
optional ``bias`` ``(out,)``; ``RMSNorm`` stores ``scale``.  Parameters are fp32
master copies; the forward pass computes in the module's compute dtype (bf16 on
the GPU, fp32 in CPU parity tests), like flax ``dtype=bf16`` modules.
"""
from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn as nn

from .. import ops


def lecun_normal_(t: torch.Tensor, fan_in: int) -> torch.Tensor:
    """Flax ``lecun_normal``: truncated normal (2 sigma) with variance 1/fan_in."""
    std = math.sqrt(1.0 / fan_in) / 0.87962566103423978
    with torch.no_grad():
        return nn.init.trunc_normal_(t, 0.0, std, -2 * std, 2 * std)


def tp_world_rank():
    """(world, rank) of the tensor-parallel group the model is built for."""
    from ..parallel.context import get_parallel_context
    pc = get_parallel_context()
    return max(pc.tp_world, 1), pc.tp_rank


class Dense(nn.Module):
    """``tp``: ``""`` replicated; ``"col"`` output features split over the
    tensor-parallel ranks (``"col2"``: the output is two equal blocks, each split);
    ``"row"`` input features split.  ``d_in`` / ``d_out`` are the full sizes."""

    def __init__(self, d_in: int, d_out: int, bias: bool = False, dtype=torch.float32, tp: str = ""):
        super().__init__()
        self.d_in, self.d_out = d_in, d_out
        W, _ = tp_world_rank()
        self.tp = tp if W > 1 else ""
        li = d_in // W if self.tp == "row" else d_in
        lo = d_out // W if self.tp in ("col", "col2") else d_out
        if self.tp and (d_in if self.tp == "row" else d_out) % (W * (2 if self.tp == "col2" else 1)):
            raise ValueError(f"Dense({d_in}, {d_out}) does not split over {W} tensor-parallel ranks")
        if self.tp == "row" and bias:
            raise ValueError("a row-parallel Dense has no bias (it would be added once per rank)")
        self.bias = nn.Parameter(torch.zeros(lo, dtype=torch.float32)) if bias else None
        if self.tp:
            # every rank draws the full matrix (same seed, same order) and keeps its piece, so the
            # initial model does not depend on the tensor-parallel layout
            from ..parallel.tp import mark_shard, shard_tensor
            _, rank = tp_world_rank()
            dim, parts = (0 if self.tp == "row" else 1), (2 if self.tp == "col2" else 1)
            full = lecun_normal_(torch.empty(d_in, d_out, dtype=dtype), d_in)
            self.kernel = nn.Parameter(shard_tensor(full, dim, parts, W, rank).clone())
            mark_shard(self.kernel, dim, parts)
            if self.bias is not None:
                mark_shard(self.bias, 0, parts)
        else:
            self.kernel = nn.Parameter(torch.empty(li, lo, dtype=dtype))
            lecun_normal_(self.kernel.data, d_in)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if ops.use_cuda(x) and x.dtype == torch.bfloat16:
            from ..ops import kernels as K
            return K.linear_multi(x, [(self.kernel, self.bias)])[0]
        return ops.linear(x, self.kernel, self.bias)


class RMSNorm(nn.Module):
    """``tp=True``: the scale of a head-split activation, split like its channels
    (the statistics then need ``parallel.tp.tp_rmsnorm``)."""

    def __init__(self, d: int, eps: float = 1e-6, tp: bool = False):
        super().__init__()
        self.eps = eps
        self.d = d
        W, _ = tp_world_rank()
        self.tp = tp and W > 1
        self.scale = nn.Parameter(torch.ones(d // W if self.tp else d, dtype=torch.float32))
        if self.tp:
            from ..parallel.tp import mark_shard
            mark_shard(self.scale, 0)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return ops.rmsnorm(x, self.scale, self.eps)


def compute_dtype_of(module: nn.Module) -> torch.dtype:
    return getattr(module, "_compute_dtype", torch.float32)
