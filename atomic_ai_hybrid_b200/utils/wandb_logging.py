"""Optional Weights & Biases logging (reference `wandb_logging.py:32-142`).

Every call is a no-op when ``wandb`` is not installed or no run is active, and
every call swallows its own exceptions, like the reference wrapper.  The same
metric keys are used (``train/*``, ``moe/*``, ``nonfinite/group_*``, ``eval/*``,
``checkpoint/*``)."""
from __future__ import annotations

from typing import Dict, Optional

_RUN = None


def init_wandb(project: str, config: Optional[Dict] = None, run_id: Optional[str] = None,
               name: Optional[str] = None) -> bool:
    global _RUN
    try:
        import wandb  # type: ignore
        _RUN = wandb.init(project=project, config=config, id=run_id, name=name, resume="allow")
        return True
    except Exception:
        _RUN = None
        return False


def log_metrics(step: int, metrics: Dict) -> None:
    if _RUN is None:
        return
    try:
        _RUN.log(metrics, step=step)
    except Exception:
        pass


def set_summary(key: str, value) -> None:
    if _RUN is None:
        return
    try:
        _RUN.summary[key] = value
    except Exception:
        pass


def log_alert(title: str, text: str, level: str = "WARN") -> None:
    print(f"[ALERT:{level}] {title}: {text}", flush=True)
    if _RUN is None:
        return
    try:
        import wandb  # type: ignore
        _RUN.alert(title=title, text=text, level=getattr(wandb.AlertLevel, level, wandb.AlertLevel.WARN))
    except Exception:
        pass


def finish() -> None:
    global _RUN
    if _RUN is None:
        return
    try:
        _RUN.finish()
    except Exception:
        pass
    _RUN = None
