"""Sharded-data-parallel communication for a ``FlatParamStore``.

The reference shards parameters and optimizer state over a 1-D mesh through
GSPMD (reference `train_setup.py:415-468`): XLA inserts an all-gather of each
parameter before use and a reduce-scatter of each gradient.  Here the layout is
explicit: every tensor has one owner rank, the fp32 gradient accumulator is
reduced onto the owners once per optimizer step, the owners update their fp32
masters, and the new compute weights (bf16 matrices, fp32 small tensors) are
gathered back to every rank, where they stay resident for all micro-steps of
the next step (a B200 holds a full bf16 copy of the benchmark models easily).

Two implementations:

* ``NcclShardComm`` -- ``reduce_scatter_tensor`` / ``all_gather_into_tensor``
  (NCCL on GPUs; emulated with ``all_reduce``/``all_gather`` on gloo for CPU tests).
* ``SymmShardComm`` (``parallel.symm``) -- gradient and compute buffers in
  CUDA-IPC peer memory; the optimizer's prepare kernel sums the owned gradient
  slice straight from the peers' buffers over NVLink and its apply kernel stores
  the updated weights into every peer's compute buffer.  Chosen by default on a
  single node with NCCL; ``AHB_SHARD_COMM=nccl`` forces the NCCL path.
"""
from __future__ import annotations

import os
from typing import Optional

import torch
import torch.distributed as dist


class NcclShardComm:
    def __init__(self, store, group: Optional[dist.ProcessGroup] = None):
        self.store = store
        self.group = group
        self.world = store.world
        self.rank = store.rank
        self.backend = dist.get_backend(group)
        self._rs_out = torch.empty(store.shard, dtype=torch.float32, device=store.device)

    def reduce_scatter_grads(self) -> None:
        st = self.store
        if self.backend == "nccl":
            dist.reduce_scatter_tensor(self._rs_out, st.grad, group=self.group)
            st.grad[st.lo:st.hi].copy_(self._rs_out)
        else:
            dist.all_reduce(st.grad, group=self.group)

    def all_gather_params(self) -> None:
        st = self.store
        if self.backend == "nccl":
            shard = st.compute[st.clo:st.chi].clone()
            dist.all_gather_into_tensor(st.compute, shard, group=self.group)
        else:
            parts = list(st.compute.view(self.world, st.cshard).unbind(0))
            shard = parts[self.rank].clone()
            dist.all_gather(parts, shard, group=self.group)


def make_shard_comm(store, group=None, kind: str = "auto"):
    kind = os.environ.get("AHB_SHARD_COMM", kind)
    backend = dist.get_backend(group)
    if kind in ("auto", "symm") and backend == "nccl" and store.device.type == "cuda":
        try:
            from .symm import SymmShardComm
            return SymmShardComm(store, group)
        except Exception as e:  # peer memory unavailable: say so, use NCCL
            if kind == "symm":
                raise
            print(f"[fsdp] peer-memory path unavailable ({e!r}); using NCCL collectives")
    return NcclShardComm(store, group)
