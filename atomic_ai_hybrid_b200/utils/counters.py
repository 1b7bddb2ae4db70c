"""Counts launches of this package's CUDA kernels (the ``gpu_launches`` figure of
``bench.py``).  Every call into the extension is counted with the number of
kernels that binding launches (1 unless listed in ``MULTI``, as a number or as a function of
the call's arguments)."""
from __future__ import annotations


class LaunchCounter:
    MULTI = {"gdn_fwd": 2, "gdn_fwd_train": 2, "gdn_bwd": 4, "gdn_bwd_saved": 2, "ssd_fwd": 2, "ssd_fwd_train": 2,
             "ssd_bwd": 4, "moe_fwd": 7, "moe_bwd": 8, "ce_online_fwd": 2, "add_rmsnorm_bwd": 2,
             "norm_gate_bwd": 2,
             # three GEMMs per row chunk: ce_online_bwd(h, W, labels, lse, ls, g, dW_acc, chunk_rows)
             "ce_online_bwd": lambda a, k: 3 * -(-a[0].shape[0] // a[7])}

    def __init__(self):
        self.count = 0
        self.on = False

    def reset(self):
        self.count = 0

    def enable(self):
        self.on = True

    def disable(self):
        self.on = False

    def add(self, name: str, args=(), kwargs=None):
        if self.on:
            n = self.MULTI.get(name, 1)
            self.count += n(args, kwargs or {}) if callable(n) else n


launch_counter = LaunchCounter()
