"""Router reset (reference `train.py:161-198`, ``_reset_router_params`` /
``_reset_router_opt_state``): re-draw every 2-D router kernel from N(0, stddev), put the
router temperatures back at their initial 10.0 and zero the optimizer moments of the
router parameters, leaving every other parameter and moment untouched.  The reference
keeps it behind ``RESET_ROUTER_ON_RESUME`` (off); here ``train.py --reset-router`` applies
it after a restore.  Prints ``[ROUTER-RESET]`` lines as the reference does."""
from __future__ import annotations

from typing import List

import torch

from ..models.moe import ROUTER_TEMP_INIT
from ..optim.schedule import path_key


@torch.no_grad()
def reset_router(trainer, seed: int = 1234, stddev: float = 0.02, verbose: bool = True) -> List[str]:
    """Applies the reset to the owned fp32 masters, the compute copies and the moments of
    every store of ``trainer``; returns the names of the parameters it changed."""
    g = torch.Generator().manual_seed(seed)
    changed = []
    stores = [(trainer.store, trainer.opt)]
    if getattr(trainer, "ep_store", None) is not None:
        stores.append((trainer.ep_store, trainer.ep_opt))
    if getattr(trainer, "xp_store", None) is not None:
        stores.append((trainer.xp_store, trainer.xp_opt))
    for st, opt in stores:
        for s in st.segs:
            key = path_key(s.name)
            if "router" not in key:
                continue
            if len(s.shape) == 2:
                new = torch.randn(s.shape, generator=g) * stddev
            elif len(s.shape) == 0 and "temp" in key:
                new = torch.full((), ROUTER_TEMP_INIT)
            else:
                continue
            new = new.to(st.device)
            st.compute_view(s).copy_(new)
            if s.owner == st.rank:
                st.master_view(s).copy_(new)
                o = s.offset - st.lo
                opt.m[o:o + s.numel].zero_()
                opt.v[o:o + s.numel].zero_()
            changed.append(s.name)
            if verbose:
                print(f"[ROUTER-RESET] {s.name} shape={tuple(s.shape)}", flush=True)
    return changed
