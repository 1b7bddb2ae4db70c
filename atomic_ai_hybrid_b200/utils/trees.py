"""Parameter-path helpers (reference `utils.py:1-59`).

``path_to_str`` lower-cases and concatenates the path keys without separator
(the form every substring rule of the reference matches against);
``collect_by_leaf_name`` gathers the per-MoE statistics of a name from the list
of stat dicts the model returns (the counterpart of flax ``sow`` collections)."""
from __future__ import annotations

from typing import Dict, List

import torch


def path_to_str(name: str) -> str:
    return name.replace(".", "").replace("/", "").lower()


def collect_by_leaf_name(stats: List[Dict[str, torch.Tensor]], target: str) -> List[torch.Tensor]:
    t = target.lower()
    return [s[k] for s in stats for k in s if k.lower() == t]
