"""The training entry loop (reference ``main_execution``, `train.py:344-1302`).

Behaviour kept from the reference:

* three checkpoint slots -- ``latest`` (time-based, every ``checkpoint_every_s``),
  ``best_train`` (when the training loss improves at a save) and ``best_val``
  (when the evaluation loss improves); resume from the newest committed step of
  ``resume_slot`` with graft-merge, then a NaN check of the restored weights;
* data resume by skipping the consumed micro-steps without reading them;
* a first-batch sanity check (token ids inside the vocabulary, labels equal to
  the inputs shifted by one);
* per-step diagnostics: global gradient norm, clip factor, per-group non-finite
  flags, parameter-clip flag; a burst guard (norm > 20 three steps running);
* non-finite steps: a snapshot (weights, optimizer state, the step's
  micro-batches and ``SNAPSHOT_META.json``) and an auto-stop after 4 in a row or
  25% of the last 15, saving ``latest`` first;
* SIGTERM / SIGINT: emergency save at the next step boundary, then exit;
* a session time budget, periodic evaluation with early stopping.

Differences by design: statistics stay on the device and are read once per
optimizer step (a few scalars), and the non-finite snapshot holds the weights
after the step (the reference copies every weight to the host before every
apply to have the pre-apply values; with ``skip_nonfinite=True`` the update is
skipped and the snapshot equals the pre-apply state).
"""
from __future__ import annotations

import json
import math
import os
import time
from dataclasses import asdict, dataclass, field
from datetime import timedelta
from typing import Dict, List, Optional

import numpy as np
import torch
import torch.distributed as dist

from .. import ops
from ..ckpt import CheckpointManager
from ..config import get_preset, load_yaml_config
from ..data import Prefetcher, dataloader_multi_source, resolve_source_files, synthetic_batches
from ..models import HybridMoEModel
from ..optim.schedule import DIAG_GROUPS
from ..utils import wandb_logging
from ..utils.health import PeerFailure, PeerHealth
from ..utils.phase_timer import PhaseTimer
from ..utils.monitor import (SESSION_TIME_BUDGET_SECONDS, BurstGuard, FaultInjector, NonFiniteMonitor,
                             StopSignals)
from .metrics import model_metrics, step_metrics
from .trainer import Trainer

CHECKPOINT_EVERY_SECONDS = 95 * 60


@dataclass
class TrainArgs:
    preset: str = "tiny"
    config_yaml: Optional[str] = None
    overrides: Dict = field(default_factory=dict)
    ckpt_root: str = "checkpoints"
    data_dir: Optional[str] = None
    data_prefixes: List[str] = field(default_factory=list)
    source_fractions: List[float] = field(default_factory=list)
    data_mode: str = "mixed"
    val_split: float = 0.05
    dataset_fraction: float = 1.0  # reference DATASET_FRACTION (global subsample, seeded)
    fraction_seed: int = 777
    seq_len: int = 512
    global_batch: int = 8          # sequences per micro-step over all data-parallel ranks
    accum_steps: int = 1
    epochs: int = 1
    max_steps: Optional[int] = None
    total_steps: Optional[int] = None
    optimizer: str = "hybrid"
    eval_every: int = 1000
    eval_batches: int = 20
    log_every: int = 10
    checkpoint_every_s: float = CHECKPOINT_EVERY_SECONDS
    session_budget_s: float = SESSION_TIME_BUDGET_SECONDS
    early_stop_patience: int = 5
    resume: bool = True
    resume_slot: str = "latest"
    # Hugging Face Hub mirror of the slots (reference RESUME_SOURCE / HF_REPO_ID): uploads
    # after each commit when a repo is named; with no local checkpoint a resume fetches
    # the slot from the model repo ("hf_model") or a storage bucket ("bucket")
    hf_repo_id: Optional[str] = None
    hf_bucket_id: Optional[str] = None
    resume_source: str = "local_only"
    hf_keep_last_n: int = 1
    wandb_project: Optional[str] = None
    impl: str = "cuda"
    cuda_graph: bool = True
    skip_nonfinite: bool = False
    seed: int = 0
    compute_dtype: str = "bf16"
    # tensor parallelism (heads split over groups of this many ranks; the ranks of a group
    # see the same batch) and expert parallelism (routed experts split over the same
    # group, or over all ranks without tensor parallelism)
    tensor_parallel: int = 1
    expert_parallel: int = 1
    remat: bool = False            # recompute every layer in the backward (activation checkpointing)
    context_parallel: int = 1      # sequence segments (parallel.cp); world / cp data-parallel replicas
    reset_router: bool = False     # re-draw the routers after a restore (reference RESET_ROUTER_ON_RESUME)
    pipeline_parallel: int = 1     # contiguous layer stages (parallel.pp); world / stages data-parallel replicas
    pipeline_schedule: str = "1f1b"  # or "gpipe"
    # AdamW moments of the rank-local parameters (expert blocks, tensor-parallel pieces) in
    # host memory: 8 bytes per such parameter off the GPU (configuration 5 needs it)
    offload_local_moments: bool = False
    # bf16 gradient accumulators for the expert-parallel experts (their own local store; each
    # micro-step's weight-gradient GEMM sums in fp32 and rounds once as it adds): 2 bytes per
    # expert parameter off the GPU, with the moments kept there (configuration 5 fits this way)
    expert_grad_bf16: bool = False


def _dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    use_cuda = torch.cuda.is_available()
    dev = torch.device("cuda", local) if use_cuda else torch.device("cpu")
    if use_cuda:
        torch.cuda.set_device(dev)
    if world > 1 and not use_cuda and "OMP_NUM_THREADS" not in os.environ:
        # CPU ranks of one host share its cores: one share each instead of all of them
        local = int(os.environ.get("LOCAL_WORLD_SIZE", world))
        torch.set_num_threads(max(1, (os.cpu_count() or 1) // max(local, 1)))
    if world > 1 and not dist.is_initialized():
        backend = "nccl" if use_cuda else "gloo"
        kw = {"device_id": dev} if use_cuda else {}
        timeout = timedelta(seconds=float(os.environ.get("AHB_PG_TIMEOUT_S", "300")))
        dist.init_process_group(backend, timeout=timeout, **kw)
    return rank, world, dev


def _to_device(b: Dict[str, torch.Tensor], dev) -> Dict[str, torch.Tensor]:
    return {k: (v.to(dev, non_blocking=True) if isinstance(v, torch.Tensor) else v) for k, v in b.items()}


def sanity_check_batch(batch: Dict[str, torch.Tensor], vocab: int) -> List[str]:
    """Reference first-batch checks (`train.py:590-618`): ids in range, label shift."""
    issues = []
    ids, lab = batch["input_ids"], batch["labels"]
    if int(ids.min()) < 0 or int(ids.max()) >= vocab:
        issues.append(f"token ids outside [0, {vocab})")
    valid = lab[:, :-1] != -100
    if valid.any() and not bool((lab[:, :-1] == ids[:, 1:])[valid].float().mean() > 0.99):
        issues.append("labels are not the inputs shifted by one")
    return issues


def _parallel_setup(args: TrainArgs, cfg, rank: int, world: int, dev):
    """Install the tensor- / expert-parallel groups; returns the data-parallel (rank,
    world) that the data loader shards over and the expert-parallel token capacity."""
    tp, ep = max(1, args.tensor_parallel), max(1, args.expert_parallel)
    if args.pipeline_parallel > 1:
        pp = args.pipeline_parallel
        if world % pp or tp > 1 or ep > 1 or args.context_parallel > 1:
            raise ValueError("pipeline parallelism needs world % stages == 0 and does not combine with "
                             "--tp / --ep / --cp")
        from ..parallel.context import ParallelContext, set_parallel_context
        set_parallel_context(ParallelContext())
        return rank // pp, world // pp, 0  # replica d = rank // stages reads its share
    if args.context_parallel > 1:
        cp = args.context_parallel
        if world % cp or tp > 1 or ep > 1:
            raise ValueError("context parallelism needs world % cp == 0 and does not combine with --tp / --ep")
        from ..parallel.cp import init_context_parallel
        init_context_parallel(dev, cp)
        return rank // cp, world // cp, 0  # replica d = rank // cp reads its share
    if tp > 1:
        if ep > 1 and ep != tp:
            raise ValueError("with tensor parallelism, expert parallelism runs over the same group (ep == tp)")
        from ..parallel.tp import init_tensor_parallel
        dp_world = world // tp
        rows = (args.global_batch // max(dp_world, 1)) * args.seq_len // tp
        init_tensor_parallel(tp, dev, expert_parallel=ep > 1, max_rows=rows, max_width=cfg.d_model)
        return rank // tp, dp_world, rows if ep > 1 else 0
    if ep > 1:
        if world % ep:
            raise ValueError(f"expert parallelism over groups of {ep} does not divide {world} ranks")
        from ..parallel.ep import init_expert_parallel
        init_expert_parallel(ep)
        return rank, world, args.global_batch // world * args.seq_len
    return rank, world, 0


TIMING_MICRO_STEPS = 30  # micro-steps timed one by one at the start of a run


def _print_memory_plan(args: TrainArgs, cfg, world: int, micro_batch: int) -> None:
    """The per-GPU memory plan of this layout (the reference prints XLA's memory analysis
    of the compiled step, `train.py:765-772`); informative only."""
    try:
        from ..utils.memplan import plan
        with torch.random.fork_rng(devices=[]):  # the planner's model leaves the generators as they were
            p = plan(cfg, world=world, micro_batch=micro_batch, seq_len=args.seq_len, tp=max(1, args.tensor_parallel),
                     ep=max(1, args.expert_parallel), cp=max(1, args.context_parallel),
                     pp=max(1, args.pipeline_parallel), accum_steps=args.accum_steps, remat=args.remat,
                     schedule=args.pipeline_schedule, local_moments_on_host=args.offload_local_moments,
                     expert_grad_bytes=2 if args.expert_grad_bf16 else 4)
        print(f"[MEMORY] plan per GPU: state {p['state_total_gb']} GB + activations ~{p['activations_gb_est']} GB "
              f"+ reserve {p['reserve_gb']} GB = {p['total_gb']} of {p['hbm_gb']} GB"
              + (f"; pinned host {p['host_pinned_gb_per_rank']} GB per rank, {p['host_pinned_gb_per_node']} GB "
                 f"per node of {p['host_ram_gb']} GB RAM" if p["host_pinned_gb_per_rank"] else "")
              + ("" if p["fits"] else "  -- DOES NOT FIT: reduce the micro-batch, enable --remat"
                 + (" or keep the moments on the device" if not p["host_fits"] else "")), flush=True)
    except Exception as e:  # the plan never stops a run
        print(f"[MEMORY] plan unavailable: {e!r}", flush=True)


def main_execution(args: TrainArgs) -> Dict:
    """Train per ``args``.  A failure on one rank is posted to the others
    (``utils.health``): they stop at their next step, or when the collective they wait in
    times out, with ``PeerFailure`` naming the failed rank."""
    rank, world, dev = _dist_setup()
    health = PeerHealth.create(rank, world)
    try:
        return _train(args, rank, world, dev, health)
    except PeerFailure:
        raise
    except Exception as e:
        if health is not None:
            failures = health.failed_peers()
            if failures:  # this rank's error follows from a peer's failure
                raise PeerFailure(failures, health.step) from e
            health.report(e)
        raise


def _train(args: TrainArgs, rank: int, world: int, dev, health: Optional[PeerHealth]) -> Dict:
    ops.set_impl(args.impl if dev.type == "cuda" else "eager")
    cfg = load_yaml_config(args.config_yaml) if args.config_yaml else get_preset(args.preset, **args.overrides)
    data_rank, data_world, ep_tokens = _parallel_setup(args, cfg, rank, world, dev)
    # one seed on every rank: the model draws each full tensor and keeps this rank's pieces
    # (tensor- and expert-parallel), so replicated weights start identical everywhere
    torch.manual_seed(args.seed)
    cdt = torch.bfloat16 if (args.compute_dtype == "bf16" and dev.type == "cuda") else torch.float32
    with torch.device(dev):
        model = HybridMoEModel(cfg, compute_dtype=cdt, remat=args.remat)

    # ---------------------------------------------------------------- data
    per_rank = args.global_batch // data_world
    if args.data_dir and args.data_prefixes:
        pairs = []
        for i, pfx in enumerate(args.data_prefixes):
            for p in resolve_source_files(args.data_dir, pfx):
                frac = args.source_fractions[i] if i < len(args.source_fractions) else 1.0
                pairs.append((p[0], p[1], frac))
    else:
        pairs = None

    mgrs = {s: CheckpointManager(args.ckpt_root, s, max_to_keep=1, rank=rank, world=world)
            for s in ("latest", "best_train", "best_val")}
    relay = None
    if args.hf_repo_id or args.hf_bucket_id or os.environ.get("HF_REPO_ID"):
        from ..ckpt.hub import HubRelay
        relay = HubRelay.create(args.hf_repo_id, args.hf_bucket_id, args.hf_keep_last_n)
    if relay is not None and rank == 0:
        for slot_name, mg in mgrs.items():
            mg.on_commit = (lambda step, meta, s=slot_name: relay.upload(
                mgrs[s].dir, s, step, str(meta.get("tag") or "")))
    if (args.resume and relay is not None and args.resume_source != "local_only"
            and all(mg.latest_step() is None for mg in mgrs.values())):
        if int(os.environ.get("LOCAL_RANK", "0")) == 0:  # one download per host
            want = args.resume_slot
            if relay.download(mgrs[want].dir, want, args.resume_source) is None and want != "latest":
                relay.download(mgrs["latest"].dir, "latest", args.resume_source)
        if world > 1:
            dist.barrier()
    steps_per_epoch = None
    if pairs is not None:
        _, _, micro_per_epoch, _ = dataloader_multi_source(pairs, args.global_batch, args.seq_len, args.val_split,
                                                           mode=args.data_mode, dataset_fraction=args.dataset_fraction,
                                                           fraction_seed=args.fraction_seed, rank=data_rank,
                                                           world=data_world, pin=False)
        steps_per_epoch = max(1, micro_per_epoch // args.accum_steps)
    total_steps = args.total_steps or (steps_per_epoch * args.epochs if steps_per_epoch else (args.max_steps or 1000))
    if args.pipeline_parallel > 1:
        from ..parallel.pp import PipelineTrainer
        trainer = PipelineTrainer(model, stages=args.pipeline_parallel, total_steps=total_steps,
                                  optimizer=args.optimizer, compute_dtype=cdt, device=dev,
                                  skip_nonfinite=args.skip_nonfinite, schedule=args.pipeline_schedule,
                                  data_parallel=world // args.pipeline_parallel)
    else:
        trainer = Trainer(model, total_steps=total_steps, optimizer=args.optimizer, compute_dtype=cdt, device=dev,
                          cuda_graph=args.cuda_graph and dev.type == "cuda", skip_nonfinite=args.skip_nonfinite,
                          ep_max_tokens=ep_tokens, offload_local_moments=args.offload_local_moments,
                          expert_grad_bf16=args.expert_grad_bf16)

    if rank == 0 and dev.type == "cuda":
        _print_memory_plan(args, cfg, world, per_rank)

    # ---------------------------------------------------------------- resume
    global_step, start_epoch = 0, 0
    best_val, best_train = math.inf, math.inf
    if args.resume:
        slot = args.resume_slot if mgrs[args.resume_slot].latest_step() is not None else None
        if slot is None:
            for s in ("latest", "best_train", "best_val"):
                if mgrs[s].latest_step() is not None:
                    slot = s
                    break
        if slot is not None:
            step = mgrs[slot].latest_step()
            meta = mgrs[slot].restore(step, trainer)
            global_step = int(meta.get("global_step", step))
            start_epoch = int(meta.get("epoch", 0))
            best_val = float(meta.get("best_val_loss", math.inf))
            best_train = float(meta.get("best_train_loss", math.inf))
            if not bool(torch.isfinite(trainer.store.master).all()):
                raise RuntimeError(f"restored weights from {slot}/{step} contain non-finite values")
            if rank == 0:
                print(f"[RESUME] {slot}/{step}: step={global_step} restored={len(meta['restored'])} "
                      f"fresh={len(meta['fresh'])}", flush=True)
            if args.reset_router:
                from .router_reset import reset_router
                reset_router(trainer, seed=args.seed + 1234, verbose=rank == 0)

    def make_stream(skip):
        if pairs is None:
            it = synthetic_batches(cfg.vocab_size, args.global_batch, args.seq_len, args.seed + skip, data_rank,
                                   data_world)
            return it, None
        it, val_f, _, _ = dataloader_multi_source(pairs, args.global_batch, args.seq_len, args.val_split,
                                                  skip_batches=skip, mode=args.data_mode,
                                                  dataset_fraction=args.dataset_fraction,
                                                  fraction_seed=args.fraction_seed, rank=data_rank, world=data_world)
        return Prefetcher(it), val_f

    train_stream, val_factory = make_stream(global_step * args.accum_steps)
    if rank == 0 and args.wandb_project:
        wandb_logging.init_for_checkpoints(args.wandb_project, args.ckpt_root, config=asdict(args),
                                           resume=args.resume, name=f"hybrid-{time.strftime('%Y%m%d-%H%M%S')}")
        for k, v in model_metrics(model).items():
            wandb_logging.set_summary(k, v)

    # ---------------------------------------------------------------- loop
    signals = StopSignals().install()
    injector = FaultInjector(rank)
    nonfin, burst = NonFiniteMonitor(), BurstGuard()
    t_start = time.time()
    last_ckpt = time.time()
    eval_no_improve, epochs_no_improve = 0, 0
    micro_seen = 0
    timer = PhaseTimer(dev)
    best_eval = math.inf  # best partial (in-epoch) validation loss
    t_epoch, epoch_tokens = time.time(), 0
    stop_reason = None
    tokens_per_step = args.global_batch * args.seq_len * args.accum_steps
    t_log, steps_since_log = time.time(), 0
    loss_hist: List[float] = []

    def save_latest(step, loss_val, asynchronous=True, tag=""):
        nonlocal best_train
        meta = {"global_step": step, "epoch": epoch, "best_val_loss": best_val, "best_train_loss": best_train,
                "train_loss": loss_val, "tag": tag}
        mgrs["latest"].save(step, trainer, meta, asynchronous=asynchronous)
        if loss_val is not None and loss_val < best_train:
            best_train = loss_val
            mgrs["latest"].finalize()
            meta["best_train_loss"] = best_train
            mgrs["best_train"].save(step, trainer, meta, asynchronous=asynchronous)
            if rank == 0:
                wandb_logging.log_metrics(step, {"checkpoint/best_train_loss": best_train})

    def save_best_val(step):
        mgrs["best_val"].save(step, trainer, {"global_step": step, "epoch": epoch, "best_val_loss": best_val,
                                              "best_train_loss": best_train})
        if rank == 0:
            print(f"[BEST_VAL] new best val loss {best_val:.4f} at step {step}", flush=True)
            wandb_logging.log_metrics(step, {"checkpoint/best_val_loss": best_val})

    def evaluate():
        if val_factory is None:
            return None
        tot, n = 0.0, 0
        for i, b in enumerate(val_factory()):
            if i >= args.eval_batches:
                break
            tot += float(trainer.eval_loss(_to_device(b, dev)))
            n += 1
        return tot / max(n, 1)

    epoch = start_epoch
    done = False
    first = True
    for epoch in range(start_epoch, args.epochs):
        for _ in range(steps_per_epoch or 10 ** 12):
            if args.max_steps is not None and global_step >= args.max_steps:
                done = True
                break
            if health is not None:
                health.check(global_step + 1)
            # generator states at the start of the step, kept for a non-finite snapshot
            rng_state = {"cpu": torch.get_rng_state()}
            if dev.type == "cuda":
                rng_state["cuda"] = torch.cuda.get_rng_state(dev)
            micro = []
            t_data = time.perf_counter()
            data_phase = timer.phase("data", host=True)
            data_phase.__enter__()
            for _m in range(args.accum_steps):
                b = next(train_stream)
                src = b.pop("_source_idx", None)
                if first:
                    issues = sanity_check_batch(b, cfg.vocab_size)
                    if issues and rank == 0:
                        print(f"[SANITY] first batch: {'; '.join(issues)}", flush=True)
                    first = False
                micro.append((_to_device(b, dev), src, b))
            if trainer.cuda_graph and (trainer._graph is None or trainer._graph_key != trainer._key(micro[0][0])):
                trainer.build_graph(micro[0][0])
            data_phase.__exit__(None, None, None)
            t_data = (time.perf_counter() - t_data) / len(micro)
            compute_phase = timer.phase("compute")
            compute_phase.__enter__()
            for db, _, _ in micro:
                if rank == 0 and micro_seen < TIMING_MICRO_STEPS:
                    # reference `train.py:837-874`: the first micro-steps timed on the host
                    # around a device synchronisation
                    if dev.type == "cuda":
                        torch.cuda.synchronize(dev)
                    t0 = time.perf_counter()
                    trainer.micro_step(db)
                    if dev.type == "cuda":
                        torch.cuda.synchronize(dev)
                    print(f"[TIMING] micro step {micro_seen}: data={t_data * 1e3:.0f}ms "
                          f"device={(time.perf_counter() - t0) * 1e3:.0f}ms (accumulating)", flush=True)
                else:
                    trainer.micro_step(db)
                micro_seen += 1
            compute_phase.__exit__(None, None, None)
            injector.before_apply(global_step + 1, trainer)

            def pre_apply_snapshot(is_finite, step=global_step + 1):
                # reference `train.py:963-993`: the parameters and optimizer state from before
                # the update of a non-finite step (all ranks reach this point together)
                if not bool(is_finite):
                    snap_dir = os.path.join(args.ckpt_root, "nonfinite_snapshots", str(step))
                    CheckpointManager(snap_dir, "state", max_to_keep=1, rank=rank, world=world).save(
                        step, trainer, {"epoch": epoch, "tag": "NONFINITE_PRE_APPLY"}, asynchronous=False)

            trainer.opt.before_finish = pre_apply_snapshot
            with timer.phase("apply"):
                info = trainer.apply(args.accum_steps)
            trainer.opt.before_finish = None
            timer.end_step()
            global_step += 1
            epoch_tokens += tokens_per_step
            if global_step == 1 and rank == 0 and dev.type == "cuda":
                print(f"[MEMORY] peak allocated after the first step: "
                      f"{torch.cuda.max_memory_allocated(dev) / 1e9:.1f} GB", flush=True)
            finite = bool(info["is_finite"])
            gnorm = float(info["global_norm"])
            loss_val = float(info["loss"])
            loss_hist.append(loss_val)
            flags = info["group_nonfinite_flags"].tolist()
            bad_groups = [g for g, f in zip(DIAG_GROUPS, flags) if f]
            if rank == 0:
                m = {"train/loss": loss_val, "train/global_grad_norm": gnorm,
                     "train/clip_factor": float(info["clip_factor"]),
                     "train/param_clip_triggered": int(bool(info["was_clipped"])),
                     "train/step_skipped_nonfinite": int(not finite)}
                m.update({f"nonfinite/group_{g}": int(g in bad_groups) for g in DIAG_GROUPS})
                wandb_logging.log_metrics(global_step, m)
            if burst.update(gnorm) and rank == 0:
                wandb_logging.log_alert("Burst guard triggered",
                                        f"global_grad_norm > 20 three steps running at step={global_step}")
            if not finite:
                snap = os.path.join(args.ckpt_root, "nonfinite_snapshots", str(global_step))
                torch.save(rng_state, os.path.join(snap, f"rng_rank{rank}.pt"))
                for i, (_, src, hb) in enumerate(micro):
                    np.save(os.path.join(snap, f"micro_{i}_rank{rank}_input_ids.npy"), hb["input_ids"].numpy())
                    np.save(os.path.join(snap, f"micro_{i}_rank{rank}_labels.npy"), hb["labels"].numpy())
                if rank == 0:
                    with open(os.path.join(snap, "SNAPSHOT_META.json"), "w") as f:
                        json.dump({"n_micro": len(micro), "global_step": global_step,
                                   "source_idx_per_micro": [s for _, s, _ in micro],
                                   "nonfinite_groups": bad_groups}, f)
            reason = nonfin.update(finite)
            if reason is not None:
                if rank == 0:
                    wandb_logging.log_alert("AUTO-STOP: frequent non-finite gradients",
                                            f"stopped at step {global_step}: {reason}", level="ERROR")
                save_latest(global_step, None, asynchronous=False, tag="AUTO_STOP_NONFINITE")
                stop_reason = "nonfinite"
                done = True
                break
            steps_since_log += 1
            phases = timer.report() if global_step % args.log_every == 0 else None  # every rank: one all-reduce
            if rank == 0 and global_step % args.log_every == 0:
                dt = time.time() - t_log
                tps = tokens_per_step * steps_since_log / max(dt, 1e-9)
                print(f"[step {global_step}] loss={loss_val:.4f} gnorm={gnorm:.3f} tok/s={tps:.0f}", flush=True)
                sm, lines, alerts = step_metrics(global_step, loss_val, trainer.last_info, best_train, tps, epoch,
                                                 cfg.num_experts)
                lines.insert(0, "phases (ms per step, max over ranks): "
                             + " ".join(f"{k}={v:.1f}" for k, v in phases.items()))
                sm.update({f"timing/{k}_ms": v for k, v in phases.items()})
                for line in lines:
                    print("           " + line, flush=True)
                for title, text in alerts:
                    wandb_logging.log_alert(title, text)
                wandb_logging.log_metrics(global_step, sm)
                t_log, steps_since_log = time.time(), 0
            if time.time() - last_ckpt >= args.checkpoint_every_s:
                save_latest(global_step, loss_val)
                last_ckpt = time.time()
            if args.eval_every and global_step % args.eval_every == 0:
                vl = evaluate()
                if vl is not None:
                    if rank == 0:
                        print(f"[EVAL] step {global_step}: val loss (partial, {args.eval_batches} batches) = "
                              f"{vl:.4f}", flush=True)
                        wandb_logging.log_metrics(global_step, {"eval/partial_val_loss": vl})
                    if vl < best_eval:
                        best_eval, eval_no_improve = vl, 0
                        if vl < best_val:
                            best_val = vl
                            save_best_val(global_step)
                    else:
                        eval_no_improve += 1
                        if eval_no_improve >= args.early_stop_patience:
                            if rank == 0:
                                wandb_logging.log_alert("Early stop", f"val loss did not improve for "
                                                        f"{args.early_stop_patience} evaluations, step {global_step}")
                            save_latest(global_step, loss_val, asynchronous=False, tag="EARLY_STOP")
                            stop_reason, done = "early_stop", True
            injector.after_step(global_step)
            if signals.requested is not None:
                save_latest(global_step, loss_val, asynchronous=False, tag="EMERGENCY_SIGNAL")
                stop_reason, done = "signal", True
            if time.time() - t_start >= args.session_budget_s:
                save_latest(global_step, loss_val, asynchronous=False, tag="SESSION_BUDGET")
                stop_reason, done = "time_budget", True
            if done:
                break
        if done:
            break
        # epoch end (reference `train.py:1237-1274`): validation, a forced save, best-val and
        # the epoch-level early stop
        if rank == 0:
            el = time.time() - t_epoch
            print(f"[EPOCH] {epoch} done: {epoch_tokens / max(el, 1e-9) / 1e6:.2f} M tokens/s", flush=True)
        t_epoch, epoch_tokens = time.time(), 0
        vl = evaluate() if val_factory is not None else None
        if rank == 0 and vl is not None:
            print(f"[EPOCH] {epoch}: mean validation loss {vl:.4f}", flush=True)
            wandb_logging.log_metrics(global_step, {"eval/epoch_val_loss": vl, "eval/epoch": epoch})
        if global_step > 0:
            save_latest(global_step, None, asynchronous=False, tag="EPOCH_END")
        if vl is not None:
            if vl < best_val:
                best_val, epochs_no_improve = vl, 0
                save_best_val(global_step)
            else:
                epochs_no_improve += 1
                if epochs_no_improve >= args.early_stop_patience:
                    stop_reason = "early_stop"
                    break
    for mg in mgrs.values():
        mg.finalize()
    if stop_reason is None and global_step > 0:
        save_latest(global_step, loss_hist[-1] if loss_hist else None, asynchronous=False, tag="FINAL")
    signals.uninstall()
    if rank == 0:
        final = {"final/global_step": global_step, "final/best_train_loss": best_train,
                 "final/best_val_loss": best_val, "final/stopped_by_nonfinite_limit": int(stop_reason == "nonfinite"),
                 "final/stopped_by_time_budget": int(stop_reason == "time_budget")}
        for k, v in final.items():
            wandb_logging.set_summary(k, v)
    trainer.close()
    wandb_logging.finish()
    summary = {"global_step": global_step, "stop_reason": stop_reason, "losses": loss_hist,
               "best_val": best_val, "best_train": best_train}
    if world > 1 and dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()
    return summary
