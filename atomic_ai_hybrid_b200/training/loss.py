"""Training loss (reference ``compute_loss``, `optimizer.py:315-430`).

``total = ce + aux_coef * sum(aux) + z_coef * sum(z) + collinearity_coef * sum(collinearity)``
where the router terms are summed over the MoE layers and ``ce`` is the
label-smoothed cross entropy of the tied LM head (mask label ``-100``).  In
evaluation (``deterministic=True``) the router terms are zero, as in the
reference.  Returns ``(total, aux_info)`` with the reference's 14 aux keys.
"""
from __future__ import annotations

from typing import Dict, List, Optional

import torch

from .. import ops

ROUTER_COLLINEARITY_COEF = 0.08


def _stack(stats: List[Dict], key: str) -> Optional[torch.Tensor]:
    vals = [s[key] for s in stats if key in s]
    return torch.stack([v.float() for v in vals]) if vals else None


def compute_loss(model, batch: Dict[str, torch.Tensor], deterministic: bool = False,
                 ce_chunk_size: int = 2048, collinearity_coef: Optional[float] = None):
    cfg = model.cfg
    hidden, stats = model(batch["input_ids"], return_hidden=True)
    labels = model.token_shard(batch["labels"]) if hasattr(model, "token_shard") else batch["labels"]
    sum_loss, sum_mask = ops.cross_entropy(hidden, labels, model.lm_weight(),
                                           cfg.label_smoothing, ce_chunk_size)
    ce = sum_loss / sum_mask.clamp_min(1.0)
    ce = torch.nan_to_num(ce, nan=0.0, posinf=1e4, neginf=0.0)
    zero = ce.new_zeros(())
    if deterministic or not stats:
        aux = z = coll = zero
    else:
        aux = _stack(stats, "aux_loss").sum()
        z = _stack(stats, "z_loss").sum()
        coll = _stack(stats, "router_collinearity").sum()
    coef = ROUTER_COLLINEARITY_COEF if collinearity_coef is None else collinearity_coef
    total = ce + cfg.router_aux_loss_coef * aux + cfg.router_z_loss_coef * z + coef * coll
    mc = _stack(stats, "router_max_cos")
    info = {
        "ce_loss": ce.detach(),
        "aux_loss": aux.detach(),
        "z_loss": z.detach(),
        "expert_utilization": _stack(stats, "expert_utilization"),
        "moe_dropped_ratio": _stack(stats, "moe_dropped_ratio"),
        "router_temp": _stack(stats, "router_temp"),
        "min_col_norm": _stack(stats, "min_col_norm"),
        "max_abs_logit_preclip": _stack(stats, "max_abs_logit_preclip"),
        "norm_x_mean": _stack(stats, "norm_x_mean"),
        "norm_x_max": _stack(stats, "norm_x_max"),
        "norm_x_min": _stack(stats, "norm_x_min"),
        "router_max_cos_per_layer": mc,
        "router_max_cos": mc.max() if mc is not None else zero,
        "assignment_frac": _stack(stats, "assignment_frac"),
    }
    return total, info
