"""Optional Weights & Biases logging (reference `wandb_logging.py:32-142`).

Every call is a no-op when ``wandb`` is not installed or no run is active, and
every call swallows its own exceptions, like the reference wrapper.  The same
metric keys are used (``train/*``, ``moe/*``, ``nonfinite/group_*``, ``eval/*``,
``checkpoint/*``)."""
from __future__ import annotations

from typing import Dict, Optional

_RUN = None


def init_wandb(project: str, config: Optional[Dict] = None, run_id: Optional[str] = None,
               name: Optional[str] = None) -> Optional[str]:
    """Start (or, with ``run_id``, continue) a run; returns its id, None without wandb."""
    global _RUN
    try:
        import wandb  # type: ignore
        _RUN = wandb.init(project=project, config=config, id=run_id, name=name, resume="allow")
        return str(getattr(_RUN, "id", None) or run_id or "") or None
    except Exception:
        _RUN = None
        return None


RUN_ID_FILE = "wandb_run_id.txt"


def init_for_checkpoints(project: str, ckpt_root: str, config: Optional[Dict] = None, resume: bool = True,
                         name: Optional[str] = None) -> Optional[str]:
    """Reference `train.py:563-588`: the run id lives in ``{ckpt_root}/wandb_run_id.txt``,
    so a restarted job that resumes from those checkpoints continues the same run (its
    curves stay continuous); a fresh start (``resume=False``) opens a new run."""
    import os
    path = os.path.join(ckpt_root, RUN_ID_FILE)
    prev = None
    if resume and os.path.exists(path):
        with open(path) as f:
            prev = f.read().strip() or None
    run_id = init_wandb(project, config=config, run_id=prev, name=name)
    if run_id is not None:
        os.makedirs(ckpt_root, exist_ok=True)
        with open(path, "w") as f:
            f.write(run_id)
    return run_id


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
