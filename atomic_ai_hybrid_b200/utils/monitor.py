"""Host-side training guards (reference `train.py:925-1035`, `train_setup.py:188-190`).

* ``NonFiniteMonitor`` -- auto-stop after ``consecutive`` non-finite steps in a
  row, or when at least ``ratio`` of the last ``window`` steps were non-finite.
* ``BurstGuard`` -- alert when the global gradient norm exceeds ``threshold``
  for ``streak`` consecutive steps.
* ``StopSignals`` -- turns SIGTERM / SIGINT into a flag the loop checks at a step
  boundary (emergency save, then exit); no collective or kernel is interrupted.
* ``FaultInjector`` -- host-side fault injection driven by environment variables,
  for tests: a NaN written into one rank's gradient at a step, an exception
  raised by one rank at a step, a signal sent to the process at a step.  Nothing
  here touches device memory outside the normal gradient buffer.
"""
from __future__ import annotations

import os
import signal
from collections import deque
from typing import Optional

NONFINITE_CONSECUTIVE_LIMIT = 4
NONFINITE_WINDOW_SIZE = 15
NONFINITE_WINDOW_RATIO = 0.25
SESSION_TIME_BUDGET_SECONDS = 9 * 3600 - 5 * 60


class NonFiniteMonitor:
    def __init__(self, consecutive: int = NONFINITE_CONSECUTIVE_LIMIT, window: int = NONFINITE_WINDOW_SIZE,
                 ratio: float = NONFINITE_WINDOW_RATIO):
        self.consecutive_limit = consecutive
        self.ratio = ratio
        self.window = deque(maxlen=window)
        self.consecutive = 0

    def update(self, finite: bool) -> Optional[str]:
        """Record one step; returns a stop reason or ``None``."""
        self.window.append(0 if finite else 1)
        self.consecutive = 0 if finite else self.consecutive + 1
        if self.consecutive >= self.consecutive_limit:
            return f"{self.consecutive} non-finite steps in a row"
        if len(self.window) >= self.window.maxlen and sum(self.window) / len(self.window) >= self.ratio:
            return f"{100 * sum(self.window) / len(self.window):.0f}% non-finite over the last {len(self.window)} steps"
        return None


class BurstGuard:
    def __init__(self, threshold: float = 20.0, streak: int = 3):
        self.threshold, self.streak_limit, self.streak = threshold, streak, 0

    def update(self, grad_norm: float) -> bool:
        self.streak = self.streak + 1 if grad_norm > self.threshold else 0
        if self.streak >= self.streak_limit:
            self.streak = 0
            return True
        return False


class StopSignals:
    def __init__(self):
        self.requested: Optional[int] = None
        self._old = {}

    def install(self):
        for sig in (signal.SIGTERM, signal.SIGINT):
            self._old[sig] = signal.getsignal(sig)
            signal.signal(sig, self._handler)
        return self

    def _handler(self, signum, frame):
        self.requested = signum

    def uninstall(self):
        for sig, h in self._old.items():
            signal.signal(sig, h)


class FaultInjector:
    """``AHB_INJECT_NAN_STEP`` / ``AHB_INJECT_NAN_RANK``: NaN in the gradient at that step;
    ``AHB_INJECT_RAISE_STEP`` / ``AHB_INJECT_RAISE_RANK``: raise RuntimeError at that step;
    ``AHB_INJECT_SIGNAL_STEP``: send SIGTERM to this process at that step."""

    def __init__(self, rank: int = 0):
        env = os.environ
        self.rank = rank
        self.nan_steps = _ints(env.get("AHB_INJECT_NAN_STEP"))
        self.nan_rank = int(env.get("AHB_INJECT_NAN_RANK", "0"))
        self.raise_step = _int(env.get("AHB_INJECT_RAISE_STEP"))
        self.raise_rank = int(env.get("AHB_INJECT_RAISE_RANK", "0"))
        self.signal_step = _int(env.get("AHB_INJECT_SIGNAL_STEP"))

    def before_apply(self, step: int, trainer) -> None:
        if step in self.nan_steps and self.rank == self.nan_rank:
            trainer.store.grad[0] = float("nan")
        if self.raise_step is not None and step == self.raise_step and self.rank == self.raise_rank:
            raise RuntimeError(f"injected failure on rank {self.rank} at step {step}")

    def after_step(self, step: int) -> None:
        if self.signal_step is not None and step == self.signal_step:
            os.kill(os.getpid(), signal.SIGTERM)


def _int(v):
    return int(v) if v not in (None, "") else None


def _ints(v):
    if not v:
        return set()
    out = set()
    for part in v.split(","):
        if "-" in part:
            a, b = part.split("-")
            out.update(range(int(a), int(b) + 1))
        else:
            out.add(int(part))
    return out
