"""One-file view of a checkpoint written by any parallel layout.

A step written by ``W`` ranks holds, per rank, the tensors that rank owns: whole tensors
(data-parallel owners, pipeline stages), blocks of routed experts (``name#experts[lo:hi]``,
expert parallelism) and tensor-parallel pieces (``name#tp[r/W,d<dim>p<parts>]``).  A
restore assembles what it needs on the fly (``ckpt.manager``); ``consolidate`` assembles
every tensor once and writes a single-rank committed step in the same format --
parameters under their flax paths in the reference's ``(in, out)`` layout and dtypes,
AdamW moments under ``mu/`` and ``nu/`` -- that any layout, a single process, or an
export to another framework can read.  The reference keeps one orbax tree per step
(`checkpointing.py:78-203`); this is the equivalent of that tree for this format.

``python -m atomic_ai_hybrid_b200.ckpt.consolidate <root> <slot> <step> <out_root>``
"""
from __future__ import annotations

import json
import os
import re
import time
from typing import Dict, Tuple

import torch

from .manager import CheckpointManager, _assemble_tp, _lookup
from .safetensors_io import save_file

_SUFFIX = re.compile(r"#(experts\[\d+:\d+\]|tp\[[^\]]*\])$")


def _base(key: str) -> str:
    return _SUFFIX.sub("", key)


def assemble(tensors: Dict[str, torch.Tensor]) -> Tuple[Dict[str, torch.Tensor], list]:
    """Every tensor whole: ``({name: tensor}, [names that could not be completed])``."""
    out: Dict[str, torch.Tensor] = {}
    missing = []
    for name in sorted({_base(k) for k in tensors}):
        if name in tensors:
            out[name] = tensors[name]
            continue
        t = _lookup(tensors, name, None)  # expert blocks
        if t is None:
            t = _assemble_tp(tensors, name)
        if t is None:
            missing.append(name)
        else:
            out[name] = t
    return out, missing


def consolidate(root: str, slot: str, step: int, out_root: str, out_slot: str = "latest") -> Dict:
    params, moments, meta = CheckpointManager(root, slot).load_tensors(step)
    p, miss_p = assemble(params)
    m, miss_m = assemble(moments)
    if miss_p:
        raise ValueError(f"step {step} of {root}/{slot} does not cover these tensors: {miss_p[:5]}")
    d = os.path.join(out_root, out_slot, str(step))
    os.makedirs(d, exist_ok=True)
    save_file(p, os.path.join(d, "params-rank0.safetensors"), {"format": "atomic_ai_hybrid_b200/params"})
    save_file(m, os.path.join(d, "opt-rank0.safetensors"), {"format": "atomic_ai_hybrid_b200/opt", "labels": "{}"})
    meta = dict(meta)
    meta.update({"world": 1, "consolidated_from": os.path.join(root, slot, str(step)),
                 "consolidated_at": time.time()})
    with open(os.path.join(d, "metadata.json"), "w") as f:
        json.dump(meta, f, indent=1)
    with open(os.path.join(d, "rank0.done"), "w") as f:
        f.write("ok")
    with open(os.path.join(d, "COMMIT"), "w") as f:
        f.write(str(step))
    return {"params": len(p), "moments": len(m), "moments_incomplete": miss_m}


if __name__ == "__main__":  # pragma: no cover
    import argparse
    ap = argparse.ArgumentParser(description="assemble a multi-rank checkpoint step into one rank's files")
    ap.add_argument("root")
    ap.add_argument("slot")
    ap.add_argument("step", type=int)
    ap.add_argument("out_root")
    a = ap.parse_args()
    print(json.dumps(consolidate(a.root, a.slot, a.step, a.out_root)))
