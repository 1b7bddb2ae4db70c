"""Per-GPU memory plan of a training layout, before anything is launched.

The reference sizes nothing ahead of time: it prints XLA's static memory analysis of the
compiled step (`train.py:765-772`).  Here the persistent state is known exactly from the
layout, so this module builds the model on the ``meta`` device under the requested
tensor- / expert-parallel split (no memory is touched), lays out the same flat stores
the trainer would build, and adds an activation estimate:

* **state** (exact): the data-parallel store holds, per parameter it covers, an fp32
  gradient accumulator and a compute copy (bf16 matrices, fp32 small tensors) in full,
  plus the fp32 master and the two optimizer moments for the owned shard only
  (``optim.store.FlatParamStore``, ``optim.hybrid.HybridOptimizer``).  Rank-local
  parameters (this rank's routed experts, its tensor-parallel pieces) sit in a store
  of their own with all five buffers in full.  With pipeline stages, a stage holds
  only its layers (the largest stage is reported) and its store is sharded over the
  stage's data-parallel replicas.
* **activations** (estimate): ``ACT_BYTES_PER_TOKEN_LAYER_D`` bytes per token, per layer,
  per model-width unit, for what the backward keeps plus the kernels' working buffers.
  The coefficient is the measured peak of the 1-GPU benchmark step (hybrid_1b,
  4 x 4096 tokens per micro-step: 167.5 GB allocated at peak) less its exact state,
  divided by tokens x layers x d_model.  With layer recomputation only each layer's
  bf16 input is kept, plus one layer's full working set.  Tensor and context
  parallelism divide the tokens a rank holds; a 1F1B stage ``s`` of ``S`` keeps up to
  ``S - s`` micro-batches (GPipe: all of them).

``python -m atomic_ai_hybrid_b200.utils.memplan --config <run file> --world 8`` (run files in
``atomic_ai_hybrid_b200/configs``) prints the plan as JSON; ``fits`` compares the total with the B200's memory.
"""
from __future__ import annotations

import argparse
import os
import json
from typing import Dict, Optional

import torch

HBM_BYTES = 183_359 * 2 ** 20          # B200 memory as nvidia-smi reports it
GPUS_PER_NODE = 8
CONTEXT_RESERVE = 2 * 10 ** 9          # CUDA context, NCCL and library workspaces
ACT_BYTES_PER_TOKEN_LAYER_D = 81.0     # calibrated on the 1-GPU benchmark step (module doc)


def _stores_bytes(module: torch.nn.Module, shard_world: int, compute_dtype: torch.dtype,
                  local_grad_bytes: int = 4, local_moments_on_host: bool = False,
                  expert_grad_bytes: Optional[int] = None) -> Dict[str, float]:
    """``local_grad_bytes``: gradient bytes per rank-local parameter; ``expert_grad_bytes``
    (default: the same) for the expert-parallel experts among them, which can keep bf16
    accumulators in a store of their own."""
    from ..optim import FlatParamStore, grad_scale_of, label_adamw_only
    from ..optim.store import is_ep_local
    named = list(module.named_parameters())
    out = {"replicated_params": 0, "local_params": 0, "master": 0.0, "grad": 0.0, "compute": 0.0,
           "optimizer": 0.0, "host_pinned": 0.0}
    meta = torch.device("meta")
    rep = [n for n, p in named if not is_ep_local(n, p)]
    loc = [n for n, p in named if is_ep_local(n, p)]
    if rep:
        st = FlatParamStore(module, label_adamw_only, grad_scale_of, shard_world, 0, compute_dtype=compute_dtype,
                            device=meta, param_filter=lambda n, p: not is_ep_local(n, p))
        out["replicated_params"] = sum(s.numel for s in st.segs)
        out["master"] += 4.0 * st.shard
        out["grad"] += 4.0 * st.numel
        out["compute"] += 2.0 * st.cnumel  # 16-bit units; an fp32 tensor takes two
        out["optimizer"] += 8.0 * st.shard
    if loc:
        st = FlatParamStore(module, label_adamw_only, grad_scale_of, 1, 0, compute_dtype=compute_dtype, device=meta,
                            param_filter=is_ep_local)
        out["local_params"] = sum(s.numel for s in st.segs)
        out["master"] += 4.0 * st.shard
        eg = local_grad_bytes if expert_grad_bytes is None else expert_grad_bytes
        n_exp = sum(s.numel for s in st.segs if getattr(s.param, "_ahb_ep_local", False))
        out["grad"] += float(local_grad_bytes) * (st.numel - n_exp) + float(eg) * n_exp
        out["compute"] += 2.0 * st.cnumel
        if not local_moments_on_host:
            out["optimizer"] += 8.0 * st.shard
        else:  # the two fp32 moments move to pinned host memory of the rank's node
            out["host_pinned"] += 8.0 * st.shard
    return out


def host_ram_bytes() -> Optional[int]:
    """Physical memory of this machine (None where the page counts are unavailable)."""
    try:
        return int(os.sysconf("SC_PAGE_SIZE")) * int(os.sysconf("SC_PHYS_PAGES"))
    except (ValueError, OSError, AttributeError):
        return None


def activation_bytes(cfg, micro_batch: int, seq_len: int, layers: int, tp: int = 1, cp: int = 1,
                     in_flight: int = 1, remat: bool = False) -> float:
    """Estimated activation + working-buffer bytes on one rank (module doc)."""
    tokens = micro_batch * seq_len / (tp * cp)
    per_layer = ACT_BYTES_PER_TOKEN_LAYER_D * cfg.d_model * tokens
    if remat:
        return in_flight * layers * 2.0 * cfg.d_model * tokens + per_layer
    return in_flight * layers * per_layer


def plan(cfg, world: int = 1, micro_batch: int = 1, seq_len: int = 4096, tp: int = 1, ep: int = 1, cp: int = 1,
         pp: int = 1, accum_steps: int = 1, remat: bool = False, schedule: str = "1f1b",
         compute_dtype: torch.dtype = torch.bfloat16, local_grad_bytes: int = 4,
         local_moments_on_host: bool = False, host_ram_gb: Optional[float] = None,
         expert_grad_bytes: Optional[int] = None) -> Dict:
    """Memory of the most loaded rank of a layout, in bytes and GB (1e9).

    With ``local_moments_on_host`` the rank-local AdamW moments live in pinned host memory:
    ``host_pinned_gb_per_rank`` and ``host_pinned_gb_per_node`` (up to 8 ranks per node) count
    them, and the layout fits only while a node's share stays within half of ``host_ram_gb``
    (default: this machine's physical memory)."""
    from ..models import HybridMoEModel
    from ..parallel.context import ParallelContext, get_parallel_context, set_parallel_context
    for n, v in (("tp", tp), ("ep", ep), ("cp", cp), ("pp", pp)):
        if world % v:
            raise ValueError(f"{n}={v} does not divide world={world}")
    saved = get_parallel_context()
    set_parallel_context(ParallelContext(tp_world=tp, tp_rank=0, ep_world=ep, ep_rank=0, dp_world=world))
    try:
        with torch.device("meta"):
            model = HybridMoEModel(cfg, compute_dtype=compute_dtype, remat=remat)
    finally:
        set_parallel_context(saved)
    if pp > 1:
        from ..parallel.pp import PipelineStage
        best = None
        for s in range(pp):
            part = PipelineStage(model, pp, s)
            b = _stores_bytes(part, world // pp, compute_dtype, local_grad_bytes, local_moments_on_host,
                              expert_grad_bytes)
            tot = b["master"] + b["grad"] + b["compute"] + b["optimizer"]
            if best is None or tot > best[0]:
                best = (tot, b, s, len(part.layer_ids))
        _, state, stage, layers = best
        in_flight = min(pp - stage, accum_steps) if schedule == "1f1b" else accum_steps
    else:
        state = _stores_bytes(model, world, compute_dtype, local_grad_bytes, local_moments_on_host,
                              expert_grad_bytes)
        layers, in_flight, stage = cfg.num_layers, 1, None
    act = activation_bytes(cfg, micro_batch, seq_len, layers, tp, cp, in_flight, remat)
    state_total = state["master"] + state["grad"] + state["compute"] + state["optimizer"]
    total = state_total + act + CONTEXT_RESERVE
    gb = lambda x: round(x / 1e9, 2)  # noqa: E731
    # pinned host memory: per rank, and for the ranks of one node (up to 8 GPUs per node); the
    # node check keeps half of the machine's RAM free for the data loader, checkpoint snapshots
    # and the OS
    ranks_per_node = min(world, GPUS_PER_NODE)
    host_node = state["host_pinned"] * ranks_per_node
    ram = host_ram_gb * 1e9 if host_ram_gb is not None else host_ram_bytes()
    host_fits = bool(host_node == 0 or (ram is not None and host_node <= 0.5 * ram))
    return {
        "layout": {"world": world, "tp": tp, "ep": ep, "cp": cp, "pp": pp, "dp": world // (tp * cp * pp),
                   "micro_batch": micro_batch, "seq_len": seq_len, "remat": remat, "stage": stage},
        "params_replicated": state["replicated_params"], "params_local": state["local_params"],
        "state_gb": {k: gb(state[k]) for k in ("master", "grad", "compute", "optimizer")},
        "state_total_gb": gb(state_total), "activations_gb_est": gb(act), "reserve_gb": gb(CONTEXT_RESERVE),
        "total_gb": gb(total), "hbm_gb": gb(HBM_BYTES),
        "host_pinned_gb_per_rank": gb(state["host_pinned"]), "host_pinned_gb_per_node": gb(host_node),
        "host_ram_gb": gb(ram) if ram is not None else None, "host_fits": host_fits,
        "fits": bool(total <= HBM_BYTES and host_fits),
    }


def main(argv: Optional[list] = None) -> Dict:
    from ..config import get_preset, load_yaml_config
    ap = argparse.ArgumentParser(description="per-GPU memory plan of a training layout")
    ap.add_argument("--config", default=None, help="YAML run file ({preset, overrides, train})")
    ap.add_argument("--preset", default="hybrid_1b")
    ap.add_argument("--world", type=int, default=None)
    ap.add_argument("--micro-batch", type=int, default=None)
    ap.add_argument("--seq-len", type=int, default=None)
    for k in ("tp", "ep", "cp", "pp"):
        ap.add_argument(f"--{k}", type=int, default=None)
    ap.add_argument("--remat", action="store_true", default=None)
    ap.add_argument("--local-grad-bytes", type=int, default=4, help="gradient bytes of rank-local parameters")
    ap.add_argument("--offload-local-moments", action="store_true", default=None,
                    help="AdamW moments of rank-local parameters in host memory")
    ap.add_argument("--expert-grad-bf16", action="store_true", default=None,
                    help="bf16 gradient accumulators for the expert-parallel experts")
    ap.add_argument("--host-ram-gb", type=float, default=None,
                    help="host memory of one node for the pinned-moment check (default: this machine's)")
    a = ap.parse_args(argv)
    train: Dict = {}
    if a.config:
        import yaml
        with open(a.config) as f:
            train = (yaml.safe_load(f) or {}).get("train", {}) or {}
        cfg = load_yaml_config(a.config)
    else:
        cfg = get_preset(a.preset)
    tp = a.tp or train.get("tensor_parallel", 1)
    ep = a.ep or train.get("expert_parallel", 1)
    cp = a.cp or train.get("context_parallel", 1)
    pp = a.pp or train.get("pipeline_parallel", 1)
    world = a.world or max(tp, ep, cp, pp)
    dp = world // (tp * cp * pp)
    gb_seqs = train.get("global_batch", 1)
    mb = a.micro_batch or max(1, gb_seqs // max(dp, 1))
    out = plan(cfg, world=world, micro_batch=mb, seq_len=a.seq_len or train.get("seq_len", 4096), tp=tp, ep=ep,
               cp=cp, pp=pp, accum_steps=train.get("accum_steps", 1),
               remat=bool(a.remat if a.remat is not None else train.get("remat", False)),
               local_grad_bytes=a.local_grad_bytes,
               local_moments_on_host=bool(a.offload_local_moments if a.offload_local_moments is not None
                                          else train.get("offload_local_moments", False)),
               host_ram_gb=a.host_ram_gb,
               expert_grad_bytes=2 if (a.expert_grad_bf16 if a.expert_grad_bf16 is not None
                                       else train.get("expert_grad_bf16", False)) else None)
    print(json.dumps(out))
    return out


if __name__ == "__main__":  # pragma: no cover
    main()
