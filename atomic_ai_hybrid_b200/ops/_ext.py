"""Loader of the in-tree sm_100a extension ``atomic_ai_hybrid_b200/_ahb_cuda*.so``.

The extension is built by ``python setup.py build_ext --inplace`` (or
``__graft_entry__.build()``).  On a machine with a GPU a missing or broken
extension is an error: the CUDA ops never fall back silently.  Calls go through
a thin proxy that counts kernel launches for the benchmark report."""
from __future__ import annotations

import importlib

from ..utils.counters import launch_counter

_EXT = None


class _Counted:
    def __init__(self, mod):
        self._mod = mod

    def __getattr__(self, name):
        fn = getattr(self._mod, name)
        if not callable(fn):
            return fn

        def call(*a, **k):
            launch_counter.add(name, a, k)
            return fn(*a, **k)
        return call


def ext():
    global _EXT
    if _EXT is None:
        try:
            mod = importlib.import_module("atomic_ai_hybrid_b200._ahb_cuda")
        except ImportError as e:  # pragma: no cover - exercised on GPU boxes only
            raise RuntimeError(
                "atomic_ai_hybrid_b200: the sm_100a extension _ahb_cuda is not built or failed to load "
                f"({e}). Run `python setup.py build_ext --inplace` in the repository root.") from e
        _EXT = _Counted(mod)
    return _EXT


def available() -> bool:
    try:
        ext()
        return True
    except RuntimeError:
        return False
