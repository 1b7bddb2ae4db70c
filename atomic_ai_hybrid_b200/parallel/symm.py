"""Data-parallel optimizer step over NVLink peer memory (one node, one process per GPU).

The store's fp32 gradient buffer and its compute buffer (bf16 matrices, fp32
small tensors) are moved into ``cudaMalloc`` allocations that every rank maps
through CUDA IPC handles.  One optimizer step is then:

1. a peer barrier: every rank's micro-steps have finished writing gradients;
2. the optimizer's prepare kernel reads its owned slice from all W gradient
   buffers and sums them while it computes the norms and flags (reduce-scatter
   fused into the first pass; ``ops.kernels.optim_prepare``);
3. Muon's Newton-Schulz on the owned matrices (local);
4. the apply kernel updates the owned shard and stores every new compute
   value into all W compute buffers (all-gather fused into the update;
   ``ops.kernels.optim_apply``);
5. a peer barrier: every rank's compute copy is complete before anyone's next
   forward, and nobody zeroes a gradient buffer a peer may still read.

The reference gets the same data movement from GSPMD: a reduce-scatter of the
accumulated gradients to the parameter sharding and an all-gather of the
parameters before use (reference `train_setup.py:415-468,583-589`).

Barrier waits are bounded (``timeout_s``); a wait that runs out records a code
in a device error word, which the host reads one step later without stalling
the stream and turns into a ``RuntimeError``.

When the optimizer runs in PyTorch ops instead of the fused kernels, the same
buffers serve a stand-alone peer reduce-scatter and a peer copy-out.
"""
from __future__ import annotations

import os
from typing import List, Optional

import torch
import torch.distributed as dist

DEFAULT_TIMEOUT_S = float(os.environ.get("AHB_SYMM_TIMEOUT", "120"))


class SymmShardComm:
    fused = True

    def __init__(self, store, group: Optional[dist.ProcessGroup] = None, timeout_s: float = DEFAULT_TIMEOUT_S):
        from ..ops._ext import ext
        self.E = E = ext()
        self.store, self.group = store, group
        self.world, self.rank = store.world, store.rank
        self.timeout_s = float(timeout_s)
        if self.world > 32:
            raise ValueError("peer-memory path supports at most 32 ranks")
        dev = store.device
        sizes = [store.grad.numel() * 4, store.compute.numel() * 2, 256]
        self._own: List[int] = []
        self._opened: List[int] = []
        try:
            for n in sizes:
                self._own.append(E.ipc_alloc(n))
            mine = torch.cat([E.ipc_handle(p) for p in self._own]).numpy().tobytes()
            allh: List[Optional[bytes]] = [None] * self.world
            dist.all_gather_object(allh, mine, group=group)
            ptrs = []
            for r in range(self.world):
                if r == self.rank:
                    ptrs.append(list(self._own))
                    continue
                row = []
                for i in range(len(sizes)):
                    h = torch.frombuffer(bytearray(allh[r][64 * i:64 * (i + 1)]), dtype=torch.uint8)
                    p = E.ipc_open(h)
                    self._opened.append(p)
                    row.append(p)
                ptrs.append(row)
        except Exception:
            self._release(free_own=True)
            raise
        self.grad_peers = torch.tensor([p[0] for p in ptrs], dtype=torch.int64, device=dev)
        self.compute_peers = torch.tensor([p[1] for p in ptrs], dtype=torch.int64, device=dev)
        self.pads = torch.tensor([p[2] for p in ptrs], dtype=torch.int64, device=dev)
        grad = E.ipc_tensor(self._own[0], store.grad.numel(), store.grad)
        compute = E.ipc_tensor(self._own[1], store.compute.numel(), store.compute)
        store.adopt_buffers(grad, compute)
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)
        self._err_host = torch.zeros(1, dtype=torch.int32, pin_memory=True)
        self._err_ev = torch.cuda.Event()
        self._err_pending = False
        self.epoch = 0
        self.closed = False
        torch.cuda.synchronize(dev)
        dist.barrier(group=group)

    # ------------------------------------------------------------ barriers
    def poll(self) -> None:
        """Raise if a barrier of an earlier step timed out (reads a copy made then)."""
        if self._err_pending:
            self._err_ev.synchronize()
            self._err_pending = False
            code = int(self._err_host[0])
            if code:
                raise RuntimeError(f"rank {self.rank}: peer barrier gave up waiting for rank {code - 100} "
                                   f"after {self.timeout_s:.0f} s")

    def barrier(self) -> None:
        self.epoch += 1
        self.E.symm_barrier(self.pads, self.rank, self.epoch, self.err, self.timeout_s)

    def _post_error_copy(self) -> None:
        self._err_host.copy_(self.err, non_blocking=True)
        self._err_ev.record()
        self._err_pending = True

    # ------------------------------------------------------------ fused step
    def begin_step(self) -> None:
        self.poll()
        self.barrier()

    def end_step(self) -> None:
        self.barrier()
        self._post_error_copy()

    # ------------------------------------------------------------ stand-alone collectives
    def reduce_scatter_grads(self) -> None:
        st = self.store
        self.poll()
        self.barrier()
        # in place: peers only ever read their own slices of this buffer, and the
        # barrier that ends all_gather_params keeps them from reading past this step
        self.E.reduce_scatter_f32(self.grad_peers, st.lo, st.grad[st.lo:st.hi])

    def all_gather_params(self) -> None:
        st = self.store
        self.E.copy_out(st.compute[st.clo:st.chi], self.compute_peers, st.clo * 2)
        self.barrier()
        self._post_error_copy()

    # ------------------------------------------------------------ teardown
    def _release(self, free_own: bool) -> None:
        for p in self._opened:
            try:
                self.E.ipc_close(p)
            except Exception:
                pass
        self._opened = []
        if free_own:
            for p in self._own:
                try:
                    self.E.ipc_free(p)
                except Exception:
                    pass
            self._own = []

    def close(self) -> None:
        """Unmap the peers' buffers.  The own buffers stay allocated (the store's
        tensors view them) until the process exits."""
        if self.closed:
            return
        self.closed = True
        torch.cuda.synchronize(self.store.device)
        self._release(free_own=False)
