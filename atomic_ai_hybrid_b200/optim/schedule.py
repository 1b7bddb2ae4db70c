"""Learning-rate schedule and parameter-group labels of the reference optimizer
(reference `optimizer.py:84-239`).

* ``lr_schedule(step)``: linear warm-up 0 -> 1 over ``max(500, 0.2*total)``
  steps, then cosine decay to ``alpha=0.1`` over the remaining steps (optax
  ``join_schedules(linear, cosine)``).
* ``resume_backoff(step)``: ramps 0.7 -> 1.0 over steps 4000..5000.
* ``label_of(path, ndim)``: the reference's ordered substring rules on the
  lower-cased, separator-free path.  Rule 2 ("norm"/"bias") catches
  ``expert_bias`` before the ``frozen`` rule, exactly as in the reference, so
  ``expert_bias`` is labelled ``adamw_nodecay``; its gradient is zero, so only the
  decoupled hook moves it.
"""
from __future__ import annotations

import math

RESUME_BACKOFF_STEPS = 5000
RESUME_LR_SCALE = 0.7

LABELS = ("muon", "lion", "adamw_decay", "adamw_nodecay", "frozen")
LABEL_ID = {n: i for i, n in enumerate(LABELS)}


class LRSchedule:
    def __init__(self, total_steps: int):
        self.total_steps = total_steps
        self.warmup = max(500, int(total_steps * 0.20))
        self.decay_steps = max(1, total_steps - self.warmup)

    def __call__(self, step: int) -> float:
        if step < self.warmup:
            return step / self.warmup
        t = min(step - self.warmup, self.decay_steps) / self.decay_steps
        cos = 0.5 * (1.0 + math.cos(math.pi * t))
        return (1.0 - 0.1) * cos + 0.1


def resume_backoff(step: int) -> float:
    ramp = 1000.0
    start = RESUME_BACKOFF_STEPS - ramp
    frac = min(max((step - start) / ramp, 0.0), 1.0)
    return RESUME_LR_SCALE + (1.0 - RESUME_LR_SCALE) * frac


def path_key(name: str) -> str:
    """Reference ``path_to_str``: lower-cased keys concatenated without separator."""
    return name.replace(".", "").replace("/", "").lower()


def label_of(name: str, ndim: int, muon_diagnostic_disable: bool = False) -> str:
    p = path_key(name)
    if "embed" in p or "lm_head" in p:
        return "adamw_decay"
    if "norm" in p or "bias" in p:
        return "adamw_nodecay"
    if "expert_bias" in p:  # unreachable (kept for parity with the reference rule list)
        return "frozen"
    if "router" in p:
        return "adamw_nodecay"
    if ndim >= 2:
        if "mamba" in p:
            return "lion"
        if muon_diagnostic_disable:
            return "adamw_nodecay"
        return "muon"
    return "lion"


def label_adamw_only(name: str, ndim: int) -> str:
    """Plain AdamW everywhere: decay on matrices, none on norms/biases/scalars."""
    p = path_key(name)
    if "norm" in p or "bias" in p or ndim < 2:
        return "adamw_nodecay"
    return "adamw_decay"


def grad_scale_of(name: str) -> float:
    """Reference apply-step gradient scales (`train_setup.py:444-452`)."""
    p = path_key(name)
    s = 1.0
    if "decay_a" in p or "a_log" in p:
        s *= 0.2
    if "router" in p:
        s *= 0.3
    return s


DIAG_GROUPS = ("gdn2", "mamba2", "mla", "moe", "muon_decay", "embed", "other")


def diag_group_of(name: str) -> str:
    """Reference ``_classify_leaf_group`` (`train_setup.py:311-322`)."""
    p = path_key(name)
    if "gdn2" in p:
        return "gdn2"
    if "mamba2" in p:
        return "mamba2"
    if "mla" in p:
        return "mla"
    if "experts_block" in p or "moe" in p or "router" in p:
        return "moe"
    if "embed" in p or "lm_head" in p:
        return "embed"
    return "other"
