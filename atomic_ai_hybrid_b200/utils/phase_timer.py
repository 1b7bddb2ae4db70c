"""Device time of the training loop's phases, reported as the max over ranks.

The reference times data, compute and apply on the host around blocking reads
(`train.py:837-874,915-917,1067-1073,1228-1232`).  Here each phase is bracketed by CUDA
events on the current stream (host clocks on a CPU run), so timing adds no
synchronisation: the events are read on logging steps, after the step's loss has been
read anyway.  ``report`` averages the phases over the steps since the last report and
takes the max over ranks with one all-reduce (every rank calls it on the same steps).
"""
from __future__ import annotations

import time
from contextlib import contextmanager
from typing import Dict, List, Optional, Tuple

import torch
import torch.distributed as dist


class PhaseTimer:
    def __init__(self, device: torch.device):
        self.cuda = device.type == "cuda"
        self.device = device
        self._pending: List[Tuple[str, object, object]] = []
        self._sums: Dict[str, float] = {}
        self._steps = 0

    @contextmanager
    def phase(self, name: str, host: bool = False):
        """Time the block: device events on the current stream, or the host clock
        (``host=True``, e.g. for data loading, which leaves the device idle)."""
        if self.cuda and not host:
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            try:
                yield
            finally:
                b.record()
                self._pending.append((name, a, b))
        else:
            t0 = time.perf_counter()
            try:
                yield
            finally:
                self._pending.append((name, t0, time.perf_counter()))

    def end_step(self) -> None:
        self._steps += 1

    def _collect(self) -> None:
        for name, a, b in self._pending:
            ms = a.elapsed_time(b) if isinstance(a, torch.cuda.Event) else (b - a) * 1e3
            self._sums[name] = self._sums.get(name, 0.0) + ms
        self._pending = []

    def report(self, group: Optional[dist.ProcessGroup] = None) -> Dict[str, float]:
        """``{phase: ms per step}`` averaged since the last report, max over the ranks."""
        for _, _, b in self._pending:
            if isinstance(b, torch.cuda.Event):
                b.synchronize()
        self._collect()
        names = sorted(self._sums)
        vals = torch.tensor([self._sums[n] / max(self._steps, 1) for n in names], dtype=torch.float64)
        if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1 and names:
            t = vals.to(self.device) if dist.get_backend(group) == "nccl" else vals
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
            vals = t.cpu()
        self._sums, self._steps = {}, 0
        return {n: float(v) for n, v in zip(names, vals)}
