"""Checkpoints keyed by the reference's parameter-tree paths
(reference `checkpointing.py:78-203`, restore `train.py:217-341`).

Layout: ``{root}/{slot}/{step}/`` holds, per rank, ``params-rank{r}.safetensors``
and ``opt-rank{r}.safetensors`` with the tensors that rank owns, ``metadata.json``
(global_step, epoch, best_val_loss, best_train_loss, timestamp, train_loss, the
optimizer step count and the world size) and a ``COMMIT`` marker written last.
A step directory without ``COMMIT`` (for instance a save interrupted by a crash)
is ignored by ``steps()``/``restore``.

* Parameter names are the flax paths (``block_0/layer_1/sublayer/gdn2/q_proj/kernel``)
  with the flax ``(in, out)`` kernel layout, stored in the reference's dtypes
  (fp32, except the routed expert weights which are bf16), so trees round-trip.
* Optimizer moments are stored as ``mu/<path>`` / ``nu/<path>`` (fp32) plus the
  step count; a checkpoint written with any world size restores on any other
  (every tensor is stored whole by its owner).
* Saves are asynchronous: owned tensors are copied into pinned host buffers on a
  side stream, and a writer thread waits for that copy and writes the files
  (the reference snapshots to host first for the same reasons).
* ``restore`` is a graft-merge: tensors whose name and shape match are loaded,
  anything new or reshaped keeps its fresh initialisation and is reported.
"""
from __future__ import annotations

import json
import os
import shutil
import threading
import time
from typing import Dict, List, Optional

import torch

from ..models.hybrid import flax_path
from .safetensors_io import load_file, save_file

SLOTS = ("latest", "best_train", "best_val")


def reference_dtype(name: str) -> torch.dtype:
    """Dtype of a tensor in the reference's tree: routed experts are bf16."""
    return torch.bfloat16 if name.split(".")[-1] in ("routed_w1", "routed_w2", "routed_w3") else torch.float32


class CheckpointManager:
    def __init__(self, root: str, slot: str = "latest", max_to_keep: int = 1, rank: int = 0, world: int = 1):
        self.dir = os.path.join(root, slot)
        self.max_to_keep = max_to_keep
        self.rank, self.world = rank, world
        self._thread: Optional[threading.Thread] = None
        self._error: Optional[BaseException] = None
        # rank 0 calls on_commit(step, metadata) from the writer after a step commits
        # (the Hub relay's upload); its failures are printed, never raised
        self.on_commit = None
        os.makedirs(self.dir, exist_ok=True)

    # ------------------------------------------------------------ listing
    def steps(self) -> List[int]:
        out = []
        if not os.path.isdir(self.dir):
            return out
        for d in os.listdir(self.dir):
            if d.isdigit() and os.path.exists(os.path.join(self.dir, d, "COMMIT")):
                out.append(int(d))
        return sorted(out)

    def latest_step(self) -> Optional[int]:
        s = self.steps()
        return s[-1] if s else None

    def step_dir(self, step: int) -> str:
        return os.path.join(self.dir, str(step))

    # ------------------------------------------------------------ save
    def save(self, step: int, trainer, metadata: Optional[Dict] = None, asynchronous: bool = True) -> None:
        self.finalize()
        st, opt = trainer.store, trainer.opt
        dev = st.device
        stream = torch.cuda.Stream() if dev.type == "cuda" else None
        params: Dict[str, torch.Tensor] = {}
        moments: Dict[str, torch.Tensor] = {}
        if stream is not None:
            stream.wait_stream(torch.cuda.current_stream())
        ctx = torch.cuda.stream(stream) if stream is not None else _null()
        with ctx:
            for store, sopt, ep in _stores(trainer):
                for s in store.owned():
                    name = _key(s, ep)
                    master = store.master_view(s)
                    params[name] = _to_host(master.to(reference_dtype(s.name)), dev)
                    o = s.offset - store.lo
                    moments[f"mu/{name}"] = _to_host(sopt.m[o:o + s.numel].view(s.shape), dev)
                    moments[f"nu/{name}"] = _to_host(sopt.v[o:o + s.numel].view(s.shape), dev)
        ev = None
        if stream is not None:
            ev = torch.cuda.Event()
            ev.record(stream)
        meta = dict(metadata or {})
        meta.update({"global_step": int(meta.get("global_step", step)), "opt_count": int(opt.count),
                     "world": self.world, "timestamp": time.time()})
        labels = {_key(s, ep): s.label for store, _, ep in _stores(trainer) for s in store.owned()}

        def write():
            try:
                if ev is not None:
                    ev.synchronize()
                d = self.step_dir(step)
                os.makedirs(d, exist_ok=True)
                save_file(params, os.path.join(d, f"params-rank{self.rank}.safetensors"),
                          {"format": "atomic_ai_hybrid_b200/params"})
                save_file(moments, os.path.join(d, f"opt-rank{self.rank}.safetensors"),
                          {"format": "atomic_ai_hybrid_b200/opt", "labels": json.dumps(labels)})
                with open(os.path.join(d, f"rank{self.rank}.done"), "w") as f:
                    f.write("ok")
                if self.rank == 0:
                    with open(os.path.join(d, "metadata.json"), "w") as f:
                        json.dump(meta, f, indent=1)
                    deadline = time.time() + 600
                    while time.time() < deadline:
                        if all(os.path.exists(os.path.join(d, f"rank{r}.done")) for r in range(self.world)):
                            break
                        time.sleep(0.05)
                    else:
                        raise TimeoutError(f"checkpoint {d}: not all ranks finished writing")
                    with open(os.path.join(d, "COMMIT"), "w") as f:
                        f.write(str(step))
                    self._prune()
                    if self.on_commit is not None:
                        try:
                            self.on_commit(step, meta)
                        except Exception as e:
                            print(f"[CKPT] after-commit hook failed for step {step}: {e!r}", flush=True)
            except BaseException as e:  # surfaced by finalize()
                self._error = e

        if asynchronous:
            self._thread = threading.Thread(target=write, daemon=True)
            self._thread.start()
        else:
            write()
            self._raise()

    def finalize(self, timeout: Optional[float] = None) -> None:
        """Wait for a pending asynchronous save (reference ``_finalize_pending_save``)."""
        if self._thread is not None:
            self._thread.join(timeout)
            self._thread = None
        self._raise()

    def _raise(self):
        if self._error is not None:
            e, self._error = self._error, None
            raise e

    def _prune(self):
        steps = self.steps()
        for s in steps[:-self.max_to_keep] if self.max_to_keep > 0 else []:
            shutil.rmtree(self.step_dir(s), ignore_errors=True)

    # ------------------------------------------------------------ restore
    def load_tensors(self, step: int):
        d = self.step_dir(step)
        if not os.path.exists(os.path.join(d, "COMMIT")):
            raise FileNotFoundError(f"{d} is not a committed checkpoint")
        params, moments = {}, {}
        for fn in sorted(os.listdir(d)):
            if fn.startswith("params-rank") and fn.endswith(".safetensors"):
                params.update(load_file(os.path.join(d, fn)))
            elif fn.startswith("opt-rank") and fn.endswith(".safetensors"):
                moments.update(load_file(os.path.join(d, fn)))
        with open(os.path.join(d, "metadata.json")) as f:
            meta = json.load(f)
        return params, moments, meta

    def restore(self, step: int, trainer, load_optimizer: bool = True) -> Dict:
        """Graft-merge restore into ``trainer``; returns the metadata plus
        ``restored``/``fresh`` name lists."""
        params, moments, meta = self.load_tensors(step)
        restored, fresh = [], []
        with torch.no_grad():
            for st, opt, ep in _stores(trainer):
                for s in st.segs:
                    name = flax_path(s.name)
                    t = _find(params, name, s, ep)
                    if t is None or tuple(t.shape) != tuple(s.shape):
                        fresh.append(name)
                        continue
                    t32 = t.to(device=st.device, dtype=torch.float32)
                    st.compute_view(s).copy_(t32)
                    if s.owner == st.rank:
                        st.master_view(s).copy_(t32)
                        o = s.offset - st.lo
                        mu, nu = _find(moments, f"mu/{name}", s, ep), _find(moments, f"nu/{name}", s, ep)
                        if load_optimizer and mu is not None and tuple(mu.shape) == tuple(s.shape):
                            # into the moments' own memory (pinned host memory when they are staged)
                            opt.m[o:o + s.numel].copy_(mu.reshape(-1).to(opt.m.device))
                            opt.v[o:o + s.numel].copy_(nu.reshape(-1).to(opt.v.device))
                    restored.append(name)
                if load_optimizer:
                    opt.count = int(meta.get("opt_count", 0))
        meta = dict(meta)
        meta["restored"], meta["fresh"] = restored, fresh
        return meta


def _stores(trainer):
    """(store, optimizer, expert_parallel) for the data-parallel store and, with
    expert parallelism, the store of this rank's experts."""
    yield trainer.store, trainer.opt, False
    if getattr(trainer, "ep_store", None) is not None:
        yield trainer.ep_store, trainer.ep_opt, True
    if getattr(trainer, "xp_store", None) is not None:  # the experts with bf16 gradient accumulators
        yield trainer.xp_store, trainer.xp_opt, True


def _expert_range(s, ep: bool):
    """Global expert rows [lo, hi) held by a segment of the expert-parallel store."""
    if not ep or not getattr(s.param, "_ahb_ep_local", False):
        return None
    from ..parallel.context import get_parallel_context
    El = s.shape[0]
    lo = get_parallel_context().ep_rank * El
    return lo, lo + El


def _tp_spec(s):
    """``(dim, parts, rank, world)`` of a tensor-parallel piece (``parallel.tp``), else None."""
    from ..parallel.tp import shard_spec
    spec = shard_spec(s.param)
    if spec is None:
        return None
    from ..parallel.context import get_parallel_context
    pc = get_parallel_context()
    if pc.tp_world <= 1:
        return None
    return spec[0], spec[1], pc.tp_rank, pc.tp_world


def _key(s, ep: bool) -> str:
    """Tensor name in the files: the flax path, plus ``#experts[lo:hi]`` for a block of
    routed experts held by one expert-parallel rank, or ``#tp[r/W,d<dim>p<parts>]`` for
    the piece of tensor-parallel rank ``r`` of ``W`` (cut along ``dim``, in ``parts``
    blocks; ``parallel.tp.shard_tensor``)."""
    name = flax_path(s.name)
    rng = _expert_range(s, ep)
    if rng is not None:
        return f"{name}#experts[{rng[0]}:{rng[1]}]"
    spec = _tp_spec(s)
    if spec is not None:
        return f"{name}#tp[{spec[2]}/{spec[3]},d{spec[0]}p{spec[1]}]"
    return name


def _find(tensors: Dict[str, torch.Tensor], name: str, s, ep: bool):
    spec = _tp_spec(s)
    if spec is not None:
        return _lookup_tp(tensors, name, spec)
    t = _lookup(tensors, name, _expert_range(s, ep))
    if t is None:  # written with tensor parallelism, restored without it
        t = _assemble_tp(tensors, name)
    return t


def _tp_pieces(tensors: Dict[str, torch.Tensor], name: str):
    """{world: {rank: (tensor, dim, parts)}} of the tensor-parallel pieces of ``name``."""
    prefix = name + "#tp["
    out: Dict[int, Dict[int, tuple]] = {}
    for key, v in tensors.items():
        if not key.startswith(prefix):
            continue
        body = key[len(prefix):-1]
        rw, _, dp = body.partition(",")
        r, w = (int(x) for x in rw.split("/"))
        dim, parts = (int(x) for x in dp[1:].split("p")) if dp else (None, None)
        out.setdefault(w, {})[r] = (v, dim, parts)
    return out


def _assemble_tp(tensors: Dict[str, torch.Tensor], name: str, dim=None, parts=None):
    """The full tensor ``name`` from the pieces of any complete tensor-parallel run."""
    from ..parallel.tp import unshard_tensors
    for w, pieces in sorted(_tp_pieces(tensors, name).items()):
        if len(pieces) != w or not all(r in pieces for r in range(w)):
            continue
        d = pieces[0][1] if pieces[0][1] is not None else dim
        pa = pieces[0][2] if pieces[0][2] is not None else parts
        if d is None:
            continue
        return unshard_tensors([pieces[r][0] for r in range(w)], d, pa)
    return None


def _lookup_tp(tensors: Dict[str, torch.Tensor], name: str, spec):
    """This rank's tensor-parallel piece of ``name``: stored directly, cut from the
    full tensor, or re-cut from the pieces of a run with another tensor-parallel size."""
    from ..parallel.tp import shard_tensor
    dim, parts, rank, world = spec
    for key in (f"{name}#tp[{rank}/{world},d{dim}p{parts}]", f"{name}#tp[{rank}/{world}]"):
        if key in tensors:
            return tensors[key]
    full = tensors.get(name)
    if full is None:
        full = _assemble_tp(tensors, name, dim, parts)
    if full is None:
        return None
    return shard_tensor(full, dim, parts, world, rank)


def _lookup(tensors: Dict[str, torch.Tensor], name: str, rng):
    """The tensor ``name`` (rows ``rng`` of it when given), assembled from expert
    blocks when the checkpoint was written with expert parallelism."""
    t = tensors.get(name if rng is None else f"{name}#experts[{rng[0]}:{rng[1]}]")
    if t is not None:
        return t
    full = tensors.get(name)
    if full is not None:
        return full if rng is None else full[rng[0]:rng[1]]
    blocks = []
    prefix = name + "#experts["
    for key, v in tensors.items():
        if key.startswith(prefix):
            lo, hi = (int(x) for x in key[len(prefix):-1].split(":"))
            blocks.append((lo, hi, v))
    if not blocks:
        return None
    blocks.sort(key=lambda b: b[0])
    n = max(b[1] for b in blocks)
    lo, hi = rng if rng is not None else (0, n)
    parts, cur = [], lo
    for b_lo, b_hi, v in blocks:
        if b_hi <= cur or b_lo >= hi:
            continue
        if b_lo > cur:
            return None  # a gap: the checkpoint does not cover these experts
        parts.append(v[cur - b_lo:min(hi, b_hi) - b_lo])
        cur = min(hi, b_hi)
    return torch.cat(parts, 0) if cur == hi else None


def _to_host(t: torch.Tensor, dev: torch.device) -> torch.Tensor:
    if dev.type != "cuda":
        return t.detach().clone()
    h = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
    h.copy_(t, non_blocking=True)
    return h


class _null:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


def make_manager(root: str, slot: str, max_to_keep: int = 1, rank: int = 0, world: int = 1) -> CheckpointManager:
    """Reference ``make_manager``: one manager per slot (latest / best_train / best_val)."""
    return CheckpointManager(root, slot, max_to_keep, rank, world)


def upload_slot(local_dir: str, repo_subdir: str, step: int, msg: str = "", keep_last_n: int = 1,
                repo_id: Optional[str] = None) -> bool:
    """Reference ``upload_slot``: mirror ``{local_dir}/{step}`` to ``{repo}/{repo_subdir}/{step}``
    and prune older steps of that slot (``ckpt.hub.HubRelay.upload``); False when no relay."""
    from .hub import HubRelay
    relay = HubRelay.create(repo_id, keep_last_n=keep_last_n)
    return relay.upload(local_dir, repo_subdir, step, msg) if relay is not None else False


def download_slot(local_dir: str, repo_subdir: str, repo_id: Optional[str] = None,
                  bucket_id: Optional[str] = None) -> Optional[int]:
    """Reference ``download_slot``: the newest step of a slot from the model repo, or from an
    HF bucket when ``bucket_id`` is given (``ckpt.hub.HubRelay.download``)."""
    from .hub import HubRelay
    relay = HubRelay.create(repo_id, bucket_id=bucket_id)
    if relay is None:
        return None
    return relay.download(local_dir, repo_subdir, "bucket" if bucket_id else "hf_model")
