"""Optimizers: the reference's hybrid Muon/Lion/AdamW on a flat parameter store."""
from .schedule import LRSchedule, label_of, label_adamw_only, grad_scale_of, resume_backoff, LABELS  # noqa: F401
from .store import FlatParamStore  # noqa: F401
from .hybrid import HybridOptimizer  # noqa: F401
