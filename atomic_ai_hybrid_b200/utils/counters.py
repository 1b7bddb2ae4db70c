"""Counts launches of this package's CUDA kernels (the ``gpu_launches`` figure of
``bench.py``).  Every call into the extension is counted with the number of
kernels that binding launches (1 unless listed in ``MULTI``)."""
from __future__ import annotations


class LaunchCounter:
    MULTI = {"gdn_fwd": 2, "gdn_fwd_train": 2, "gdn_bwd": 4, "gdn_bwd_saved": 2, "ssd_fwd": 2, "ssd_fwd_train": 2,
             "ssd_bwd": 4, "moe_fwd": 7, "moe_bwd": 8, "ce_fused_fwd": 2, "ce_fused_bwd": 2, "add_rmsnorm_bwd": 2,
             "norm_gate_bwd": 2}

    def __init__(self):
        self.count = 0
        self.on = False

    def reset(self):
        self.count = 0

    def enable(self):
        self.on = True

    def disable(self):
        self.on = False

    def add(self, name: str):
        if self.on:
            self.count += self.MULTI.get(name, 1)


launch_counter = LaunchCounter()
