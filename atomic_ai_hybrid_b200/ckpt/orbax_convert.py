"""Convert a checkpoint written by the reference (orbax ``{"params", "opt_state"}``
trees, reference `checkpointing.py:78-203`) into this framework's checkpoint layout.

The parameter tree keeps its flax paths (``block_0/layer_1/sublayer/gdn2/q_proj/kernel``)
and the ``(in, out)`` kernel layout, which are the names and shapes this framework
stores (``ckpt.manager``), so parameters map one to one.  The optax state is a chain
``(clip state, MultiTransformState(inner_states={label: MaskedState(inner_state=...)}))``
whose AdamW / Lion states hold ``mu`` / ``nu`` trees shaped like the parameters, with
empty (masked) leaves for parameters of other labels; every non-empty ``mu`` / ``nu``
leaf becomes ``mu/<path>`` / ``nu/<path>``, and the largest ``count`` is the step count.

``convert_tree`` works on an already restored tree (nested dicts / lists / tuples of
arrays) and needs nothing beyond numpy; ``convert_orbax_dir`` restores the tree with
orbax, which must be installed for that part.
"""
from __future__ import annotations

import json
import os
import time
from typing import Any, Dict, Iterator, Optional, Tuple

import numpy as np
import torch

from .manager import reference_dtype
from .safetensors_io import save_file


def _children(node) -> Iterator[Tuple[str, Any]]:
    if isinstance(node, dict):
        yield from ((str(k), v) for k, v in node.items())
    elif hasattr(node, "_asdict"):  # NamedTuple states restored with their types
        yield from node._asdict().items()
    elif isinstance(node, (list, tuple)):
        yield from ((str(i), v) for i, v in enumerate(node))


def _is_array(x) -> bool:
    return hasattr(x, "shape") and hasattr(x, "dtype") and not isinstance(x, (dict, list, tuple))


def flatten(tree, prefix: str = "") -> Dict[str, Any]:
    """``{"a": {"b": x}}`` -> ``{"a/b": x}`` over arrays (empty masked leaves dropped)."""
    out: Dict[str, Any] = {}
    if _is_array(tree):
        if tree.size > 0 or tree.shape == ():
            out[prefix] = tree
        return out
    for k, v in _children(tree):
        out.update(flatten(v, f"{prefix}/{k}" if prefix else k))
    return out


def _moments(opt_state, names) -> Tuple[Dict[str, Any], Dict[str, Any], int]:
    """Every ``mu`` / ``nu`` sub-tree whose leaves are parameter paths; the largest count."""
    mu: Dict[str, Any] = {}
    nu: Dict[str, Any] = {}
    count = 0

    def walk(node):
        nonlocal count
        for k, v in _children(node):
            if k in ("mu", "nu"):
                for path, arr in flatten(v).items():
                    if path in names and tuple(arr.shape) == tuple(names[path]):
                        (mu if k == "mu" else nu).setdefault(path, arr)
            elif k == "count" and _is_array(v):
                count = max(count, int(np.asarray(v).reshape(-1)[0]))
            else:
                walk(v)

    walk(opt_state)
    return mu, nu, count


def convert_tree(tree: Dict[str, Any], dst_root: str, step: int, slot: str = "latest",
                 metadata: Optional[Dict] = None) -> Dict[str, int]:
    """Write ``tree`` (``{"params": ..., "opt_state": ...}``, or the parameter tree alone)
    as a committed single-rank checkpoint ``{dst_root}/{slot}/{step}``."""
    params_tree = tree.get("params", tree) if isinstance(tree, dict) else tree
    flat = flatten(params_tree)
    # a flax module tree restored whole nests its variables under "params"
    if all(k.startswith("params/") for k in flat):
        flat = {k[len("params/"):]: v for k, v in flat.items()}
    names = {k: tuple(v.shape) for k, v in flat.items()}
    params = {k: torch.from_numpy(np.asarray(v, dtype=np.float32)).to(reference_dtype(k.replace("/", ".")))
              for k, v in flat.items()}
    moments: Dict[str, torch.Tensor] = {}
    count = 0
    if isinstance(tree, dict) and tree.get("opt_state") is not None:
        mu, nu, count = _moments(tree["opt_state"], names)
        moments.update({f"mu/{k}": torch.from_numpy(np.asarray(v, dtype=np.float32)) for k, v in mu.items()})
        moments.update({f"nu/{k}": torch.from_numpy(np.asarray(v, dtype=np.float32)) for k, v in nu.items()})
    d = os.path.join(dst_root, slot, str(step))
    os.makedirs(d, exist_ok=True)
    save_file(params, os.path.join(d, "params-rank0.safetensors"), {"format": "atomic_ai_hybrid_b200/params"})
    save_file(moments, os.path.join(d, "opt-rank0.safetensors"),
              {"format": "atomic_ai_hybrid_b200/opt", "labels": json.dumps({})})
    meta = dict(metadata or {})
    meta.update({"global_step": int(meta.get("global_step", step)), "opt_count": int(meta.get("opt_count", count)),
                 "world": 1, "timestamp": time.time(), "converted_from": "orbax"})
    with open(os.path.join(d, "metadata.json"), "w") as f:
        json.dump(meta, f, indent=1)
    with open(os.path.join(d, "rank0.done"), "w") as f:
        f.write("ok")
    with open(os.path.join(d, "COMMIT"), "w") as f:
        f.write(str(step))
    return {"params": len(params), "moments": len(moments), "opt_count": int(meta["opt_count"])}


def convert_orbax_dir(src: str, dst_root: str, step: Optional[int] = None, slot: str = "latest") -> Dict[str, int]:
    """Restore the reference's orbax checkpoint at ``src`` (a step directory, or a
    manager directory with ``step``) and write it with ``convert_tree``."""
    try:
        import orbax.checkpoint as ocp
    except ImportError as e:  # pragma: no cover - orbax is not part of this image
        raise RuntimeError("converting an orbax checkpoint needs the orbax-checkpoint package") from e
    path = os.path.join(src, str(step)) if step is not None else src
    for sub in ("default", "state", ""):
        cand = os.path.join(path, sub) if sub else path
        if os.path.isdir(cand):
            try:
                tree = ocp.PyTreeCheckpointer().restore(cand)
                break
            except Exception:
                continue
    else:
        raise FileNotFoundError(f"no orbax tree under {path}")
    meta = {}
    for cand in (os.path.join(path, "metadata.json"), os.path.join(src, "metadata.json")):
        if os.path.exists(cand):
            with open(cand) as f:
                meta = json.load(f)
            break
    s = int(meta.get("global_step", step if step is not None else 0))
    return convert_tree(tree, dst_root, s, slot=slot, metadata=meta)


if __name__ == "__main__":  # pragma: no cover
    import argparse
    ap = argparse.ArgumentParser(description="reference (orbax) checkpoint -> this framework's layout")
    ap.add_argument("src")
    ap.add_argument("dst_root")
    ap.add_argument("--step", type=int, default=None)
    ap.add_argument("--slot", default="latest")
    a = ap.parse_args()
    print(json.dumps(convert_orbax_dir(a.src, a.dst_root, a.step, a.slot)))
