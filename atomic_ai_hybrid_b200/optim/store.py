"""Flat parameter store: fp32 master weights, fp32 gradient accumulators and the
compute copies of a model, laid out for fused sharded updates.

Layout
------
Every parameter tensor is owned by exactly one rank (greedy size balancing over
the ``world`` ranks, whole tensors only, so a matrix-wise optimizer such as Muon
sees complete matrices on its owner).  Two flat index spaces exist:

* the *state space* (fp32 elements): gradient accumulator, master weights and
  optimizer moments.  Rank ``r`` owns ``[r*S, (r+1)*S)``.
* the *compute space* (16-bit units): the weights the forward/backward pass
  reads.  Matrices are stored as bf16 (one unit per element); small tensors (norm
  scales, biases, per-head scalars, the router) stay fp32 (two units per
  element, viewed as fp32), because the reference computes with them in fp32.
  Rank ``r`` owns ``[r*CS, (r+1)*CS)``.

Per-rank ranges are padded to the largest rank total, so the gradient
reduce-scatter, the update and the parameter all-gather each move one
equal-sized slice per rank.  The gradient buffer is full size on every rank;
master and moments hold only the owned shard.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Dict, List, Optional

import torch
import torch.nn as nn

ALIGN = 64


@dataclass
class Seg:
    name: str
    shape: tuple
    numel: int
    offset: int          # state-space offset (fp32 elements)
    coff: int            # compute-space offset (16-bit units)
    owner: int
    label: str
    fp32: bool           # compute copy is fp32
    grad_scale: float
    param: nn.Parameter

    @property
    def cunits(self) -> int:
        return self.numel * (2 if self.fp32 else 1)


def _round(n: int, a: int = ALIGN) -> int:
    return (n + a - 1) // a * a


def default_keep_fp32(name: str, p: torch.Tensor) -> bool:
    return p.ndim < 2 or name.endswith("router")


def is_ep_local(name: str, p: torch.Tensor) -> bool:
    """Parameters that differ between ranks: this rank's block of routed experts
    (expert parallelism) or its piece of a tensor-parallel weight.  They are not
    reduced or gathered across the data-parallel ranks of the main store."""
    return bool(getattr(p, "_ahb_ep_local", False) or getattr(p, "_ahb_tp_shard", None) is not None)


class FlatParamStore:
    def __init__(self, model: nn.Module, label_fn: Callable[[str, int], str],
                 grad_scale_fn: Callable[[str], float], world: int = 1, rank: int = 0,
                 compute_dtype: torch.dtype = torch.bfloat16, device=None,
                 keep_fp32: Callable[[str, torch.Tensor], bool] = default_keep_fp32,
                 param_filter: Optional[Callable[[str, torch.Tensor], bool]] = None,
                 grad_dtype: torch.dtype = torch.float32):
        # ``grad_dtype`` bf16: 16-bit gradient accumulators (each weight-gradient GEMM sums in
        # fp32 and rounds once as it adds); only for stores whose gradients come from kernels
        # that accumulate into bf16 (the expert-parallel experts)
        if grad_dtype not in (torch.float32, torch.bfloat16):
            raise ValueError(f"gradient accumulators are fp32 or bf16, not {grad_dtype}")
        self.world, self.rank = world, rank
        self.compute_dtype = compute_dtype
        named = [(n, p) for n, p in model.named_parameters() if param_filter is None or param_filter(n, p)]
        self.device = device = device or named[0][1].device
        all32 = compute_dtype == torch.float32
        fp32 = [all32 or keep_fp32(n, p) for n, p in named]
        # -- owners: largest first onto the least-loaded rank
        order = sorted(range(len(named)), key=lambda i: -named[i][1].numel())
        load = [0] * world
        cload = [0] * world
        owner = [0] * len(named)
        for i in order:
            r = min(range(world), key=lambda j: load[j])
            owner[i] = r
            load[r] += _round(named[i][1].numel())
            cload[r] += _round(named[i][1].numel() * (2 if fp32[i] else 1))
        self.shard = _round(max(load), 128)
        self.cshard = _round(max(cload), 128)
        self.numel = self.shard * world
        self.cnumel = self.cshard * world
        cur = [r * self.shard for r in range(world)]
        ccur = [r * self.cshard for r in range(world)]
        self.segs: List[Seg] = []
        for i, (n, p) in enumerate(named):
            r = owner[i]
            s = Seg(n, tuple(p.shape), p.numel(), cur[r], ccur[r], r, label_fn(n, p.ndim), fp32[i],
                    grad_scale_fn(n), p)
            self.segs.append(s)
            cur[r] += _round(s.numel)
            ccur[r] += _round(s.cunits)
        self.by_name: Dict[str, Seg] = {s.name: s for s in self.segs}
        self.lo, self.hi = rank * self.shard, (rank + 1) * self.shard
        self.clo, self.chi = rank * self.cshard, (rank + 1) * self.cshard
        half = torch.float32 if all32 else compute_dtype
        self.half_dtype = torch.bfloat16 if half == torch.float32 else half
        self.master = torch.zeros(self.shard, dtype=torch.float32, device=device)
        self.grad = torch.zeros(self.numel, dtype=grad_dtype, device=device)
        self.compute = torch.zeros(self.cnumel, dtype=self.half_dtype, device=device)
        self._hooks = []
        for s in self.segs:
            src = s.param.detach().to(device=device, dtype=torch.float32).reshape(-1)
            if s.owner == rank:
                self.master[s.offset - self.lo:s.offset - self.lo + s.numel].copy_(src)
            self.compute_view(s).copy_(src.view(s.shape))
            self._rebind(s)

    def adopt_buffers(self, grad: torch.Tensor, compute: torch.Tensor) -> None:
        """Move the gradient and compute buffers into caller-provided memory (e.g.
        peer-mapped allocations) and rebind every parameter to it."""
        assert grad.shape == self.grad.shape and compute.shape == self.compute.shape
        grad.copy_(self.grad)
        compute.copy_(self.compute)
        self.grad, self.compute = grad, compute
        for h in self._hooks:
            h.remove()
        self._hooks = []
        for s in self.segs:
            self._rebind(s)

    # ------------------------------------------------------------------ views
    def compute_view(self, s: Seg) -> torch.Tensor:
        raw = self.compute[s.coff:s.coff + s.cunits]
        if s.fp32:
            return raw.view(torch.float32).view(s.shape)
        return raw.view(s.shape)

    def _rebind(self, s: Seg) -> None:
        p = s.param
        p.data = self.compute_view(s)
        if not p.requires_grad:
            return
        g = self.grad_view(s)
        p._ahb_grad_acc = g
        if s.fp32 and g.dtype == torch.float32:
            p.grad = g
        else:  # autograd's gradient is added into the accumulator (bf16 ones round here)
            def hook(param, g=g):
                if param.grad is not None:
                    g.add_(param.grad)
                    param.grad = None
            self._hooks.append(p.register_post_accumulate_grad_hook(hook))

    def grad_view(self, s: Seg) -> torch.Tensor:
        return self.grad[s.offset:s.offset + s.numel].view(s.shape)

    def master_view(self, s: Seg) -> torch.Tensor:
        assert s.owner == self.rank
        o = s.offset - self.lo
        return self.master[o:o + s.numel].view(s.shape)

    def owned(self) -> List[Seg]:
        return [s for s in self.segs if s.owner == self.rank]

    def zero_grad(self) -> None:
        self.grad.zero_()
        direct = self.grad.dtype == torch.float32  # fp32 parameters bound to their accumulators
        for s in self.segs:
            if s.fp32 and direct and s.param.requires_grad:
                s.param.grad = self.grad_view(s)

    def publish_owned(self) -> None:
        """Write the owned fp32 masters into the local compute copy."""
        for s in self.owned():
            self.compute_view(s).copy_(self.master_view(s))

    def full_state_dict(self) -> Dict[str, torch.Tensor]:
        """fp32 copies of every parameter read from the (gathered) compute buffer;
        exact for fp32 tensors, bf16-rounded for matrices unless owned."""
        out = {}
        for s in self.segs:
            if s.owner == self.rank:
                out[s.name] = self.master_view(s).clone()
            else:
                out[s.name] = self.compute_view(s).float().clone()
        return out
