"""Failure notices between the ranks of one job, through the rendezvous store.

The reference runs one SPMD program on a TPU slice and has no notion of a failed
rank (`train.py:344-1302`); a data-parallel job over processes needs one.  When a rank's
training loop raises, it records ``{rank, step, error}`` under its own key in the
process group's key-value store (the TCP store every rank already talks to) and bumps
a failure counter.  The other ranks read the counter (one store round trip) at the
start of every step, before any collective of that step, and stop with ``PeerFailure``
naming the rank, its step and its error.  A rank that is already inside a collective
when the peer fails is ended by the process group's timeout; its error is then
re-raised as ``PeerFailure`` with the same details, so every rank reports the root
cause instead of a bare timeout.

Nothing here touches a GPU: the notice travels over the host network only.
"""
from __future__ import annotations

import json
import time
from typing import Dict, List, Optional

import torch.distributed as dist

_PREFIX = "ahb_health"


class PeerFailure(RuntimeError):
    """Another rank of the job failed; ``failures`` holds its notices."""

    def __init__(self, failures: List[Dict], step: Optional[int] = None):
        self.failures = failures
        desc = "; ".join(f"rank {f['rank']} at step {f['step']}: {f['error']}" for f in failures)
        where = f" (this rank at step {step})" if step is not None else ""
        super().__init__(f"peer failure{where}: {desc}")


class PeerHealth:
    def __init__(self, store, rank: int, world: int):
        self.store, self.rank, self.world = store, rank, world
        self.step = 0

    @classmethod
    def create(cls, rank: int, world: int) -> Optional["PeerHealth"]:
        """The notice board of the default process group, or None for one rank / no store."""
        if world <= 1 or not dist.is_initialized():
            return None
        try:
            store = dist.distributed_c10d._get_default_store()
        except Exception:  # a process group created without a store
            return None
        return cls(store, rank, world)

    def _key(self, rank: int) -> str:
        return f"{_PREFIX}/failed/{rank}"

    def report(self, error: BaseException | str) -> None:
        """Record this rank's failure (best effort: the store may be gone already)."""
        note = {"rank": self.rank, "step": self.step, "error": repr(error)[:500], "time": time.time()}
        try:
            self.store.set(self._key(self.rank), json.dumps(note))
            self.store.add(f"{_PREFIX}/count", 1)
        except Exception:
            pass

    def failed_peers(self) -> List[Dict]:
        """Notices of the other ranks (empty when none failed or the store is unreachable)."""
        try:
            if self.store.add(f"{_PREFIX}/count", 0) == 0:
                return []
            out = []
            for r in range(self.world):
                if r != self.rank and self.store.check([self._key(r)]):
                    out.append(json.loads(self.store.get(self._key(r))))
            return out
        except Exception:
            return []

    def check(self, step: int) -> None:
        """Start of a step: raise ``PeerFailure`` if another rank has failed."""
        self.step = step
        failures = self.failed_peers()
        if failures:
            raise PeerFailure(failures, step)
