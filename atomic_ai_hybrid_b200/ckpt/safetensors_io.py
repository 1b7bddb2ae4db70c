"""Minimal reader/writer for the safetensors file format.

Layout: 8-byte little-endian header length, a JSON header mapping tensor names
to ``{"dtype", "shape", "data_offsets": [begin, end]}`` (plus an optional
``"__metadata__"`` string map), then the raw little-endian tensor bytes.  The
``safetensors`` package is not part of this image, so the format is written
directly; files are readable by any safetensors implementation.
"""
from __future__ import annotations

import json
import os
import struct
from typing import Dict, Optional, Tuple

import numpy as np
import torch

_DT = {torch.float32: "F32", torch.bfloat16: "BF16", torch.float16: "F16", torch.int64: "I64",
       torch.int32: "I32", torch.uint8: "U8", torch.float64: "F64", torch.bool: "BOOL"}
_RDT = {v: k for k, v in _DT.items()}


def save_file(tensors: Dict[str, torch.Tensor], path: str, metadata: Optional[Dict[str, str]] = None) -> None:
    header = {}
    off = 0
    items = []
    for name in sorted(tensors):
        t = tensors[name].detach().contiguous().cpu()
        nbytes = t.numel() * t.element_size()
        header[name] = {"dtype": _DT[t.dtype], "shape": list(t.shape), "data_offsets": [off, off + nbytes]}
        items.append(t)
        off += nbytes
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    hb = json.dumps(header, separators=(",", ":")).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for t in items:
            f.write(t.reshape(-1).view(torch.uint8).numpy().tobytes() if t.numel() else b"")
        f.flush()
        os.fsync(f.fileno())
    os.replace(tmp, path)


def read_header(path: str) -> Tuple[dict, int]:
    with open(path, "rb") as f:
        raw = f.read(8)
        if len(raw) != 8:
            raise ValueError(f"{path}: truncated safetensors header")
        (n,) = struct.unpack("<Q", raw)
        hb = f.read(n)
        if len(hb) != n:
            raise ValueError(f"{path}: truncated safetensors header")
    return json.loads(hb), 8 + n


def load_file(path: str) -> Dict[str, torch.Tensor]:
    header, base = read_header(path)
    size = os.path.getsize(path)
    out = {}
    buf = np.memmap(path, dtype=np.uint8, mode="r")
    for name, info in header.items():
        if name == "__metadata__":
            continue
        b, e = info["data_offsets"]
        if base + e > size:
            raise ValueError(f"{path}: truncated data for {name}")
        raw = torch.from_numpy(np.array(buf[base + b:base + e]))
        dt = _RDT[info["dtype"]]
        out[name] = raw.view(dt).reshape(info["shape"]) if raw.numel() else torch.empty(info["shape"], dtype=dt)
    return out


def load_metadata(path: str) -> Dict[str, str]:
    header, _ = read_header(path)
    return header.get("__metadata__", {})
