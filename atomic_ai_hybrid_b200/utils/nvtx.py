"""NVTX ranges for external timeline tools (``AHB_NVTX=1``): one range per layer of
the forward, per micro-step and per optimizer step.  Host-side only, so they cost
nothing on the device and survive CUDA-graph capture (the captured kernels keep
the ranges of the capture).  The reference has no profiler hooks; its timing is
host ``perf_counter`` around data / compute / apply (`train.py:837-874`)."""
from __future__ import annotations

import contextlib
import os

import torch

ON = os.environ.get("AHB_NVTX", "0") == "1"


@contextlib.contextmanager
def nvtx_range(name: str):
    if ON and torch.cuda.is_available():
        torch.cuda.nvtx.range_push(name)
        try:
            yield
        finally:
            torch.cuda.nvtx.range_pop()
    else:
        yield
