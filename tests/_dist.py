"""Helpers for the multi-process CPU tests (gloo ranks as spawned processes).

* ``free_port``: a rendezvous port from a range private to this pytest-xdist worker, checked
  free by binding it, so concurrent workers never draw the same port.
* ``threads_per_rank``: one share of the cores per rank, counting every concurrent xdist
  worker's ranks, so a loaded run is not oversubscribed several times over.
* ``collect``: results from the ranks' queue, failing at once (with the rank's exit code) when
  a rank dies without reporting, and waiting at most ``timeout`` seconds scaled by the machine's
  load (a slow but live run is not cut off early).
"""
from __future__ import annotations

import itertools
import os
import queue
import socket
import time

_counter = itertools.count()


def _worker_index() -> int:
    w = os.environ.get("PYTEST_XDIST_WORKER", "gw0")
    try:
        return int(w.lstrip("gw"))
    except ValueError:
        return 0


def free_port() -> int:
    base = 30000 + 400 * (_worker_index() % 60) + (os.getpid() % 7) * 50
    for _ in range(400):
        p = base + next(_counter) % 400
        s = socket.socket()
        try:
            s.bind(("127.0.0.1", p))
            return p
        except OSError:
            continue
        finally:
            s.close()
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def threads_per_rank(world: int) -> int:
    workers = int(os.environ.get("PYTEST_XDIST_WORKER_COUNT", "1") or 1)
    return max(1, (os.cpu_count() or 2) // max(1, world * workers))


def load_factor() -> float:
    try:
        return max(1.0, os.getloadavg()[0] / (os.cpu_count() or 1))
    except OSError:
        return 1.0


def collect(procs, q, n: int, timeout: float = 300.0):
    """``n`` results from ``q``; raises if a rank exits without one or the deadline passes."""
    out = []
    deadline = time.monotonic() + timeout * load_factor()
    while len(out) < n:
        try:
            out.append(q.get(timeout=2.0))
            continue
        except queue.Empty:
            pass
        for r, p in enumerate(procs):
            if p.exitcode not in (None, 0):
                raise RuntimeError(f"rank {r} exited with code {p.exitcode} before reporting")
        if all(p.exitcode is not None for p in procs) and q.empty():
            raise RuntimeError(f"all ranks exited with {len(out)} of {n} results")
        if time.monotonic() > deadline:
            # extend while the machine is busier than when the wait began
            if time.monotonic() > deadline + timeout * (load_factor() - 1.0):
                raise TimeoutError(f"{len(out)} of {n} results after {timeout * load_factor():.0f} s")
    return out
