"""Training-throughput benchmark (train tokens/sec, whole job, max over ranks).

Contract: ``python bench.py --gpus N --steps K --warmup W`` (torchrun for N>1)
runs the flagship training step -- the hybrid GDN-2/Mamba2 MoE LM of the
benchmark's config 3 (d_model 2048, 24 layers alternating GDN 16x128 and Mamba2
32x64 with d_state 128, 32 routed SwiGLU experts top-4 of hidden 1024 plus one
shared expert, vocab 50304, seq 4096), bf16 compute, fp32 master weights,
AdamW -- on synthetic tokens with random-init weights, and rank 0 prints one
JSON line.  Scaling is weak: every GPU processes ``--seqs-per-gpu`` sequences per
optimizer step (32 by default, i.e. global batch 256 at 8 GPUs).

``--impl cuda`` (default) runs the sm_100a kernels; ``--impl eager`` runs the
unfused PyTorch + cuBLAS + NCCL baseline of the identical model; ``--impl
reference`` would run the reference project itself, which cannot be installed
on this image (its JAX/Flax/Optax/Orbax stack is absent and it has no build
metadata), so that arm prints its ``unavailable`` line.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
# the baseline of this metric: the unfused PyTorch + cuBLAS + NCCL implementation of the same
# model (`--impl eager`) measured on 1 x B200, hybrid_1b, seq 4096, 32 sequences per step; the
# reference publishes no figure for it
EAGER_BASELINE_TOKS = 508.7
sys.path.insert(0, HERE)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="cuda", choices=["cuda", "eager", "reference"])
    ap.add_argument("--model", default="hybrid_1b")
    ap.add_argument("--seq-len", type=int, default=4096)
    ap.add_argument("--seqs-per-gpu", type=int, default=32)
    ap.add_argument("--micro-batch", type=int, default=4)
    ap.add_argument("--layers", type=int, default=None, help="override num_layers (debug only; invalid for the bench)")
    ap.add_argument("--optimizer", default="adamw", choices=["adamw", "hybrid"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-scan-ops", action="store_true",
                    help="skip the scan-operator figures measured after the timed region")
    ap.add_argument("--no-graph", action="store_true", help="disable CUDA-graph capture of the micro-step")
    ap.add_argument("--ep", type=int, default=1,
                    help="expert-parallel ranks (1 or the number of GPUs): routed experts split over the GPUs")
    ap.add_argument("--expert-grad-bf16", action="store_true",
                    help="bf16 gradient accumulators for the expert-parallel experts (the long-context layout)")
    ap.add_argument("--remat", action="store_true", help="recompute each layer in the backward")
    ap.add_argument("--tp", type=int, default=1,
                    help="tensor-parallel ranks (heads split, tokens split between the mixers); each group of "
                         "--tp GPUs trains on --seqs-per-gpu x --tp sequences per step")
    return ap.parse_args()


class ClockSampler:
    """Samples SM clocks / throttle reasons with nvidia-smi during the timed region."""

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = f"/tmp/ahb_clocks_{os.getpid()}.csv"

    def _gpu_id(self) -> str:
        """nvidia-smi's name for this process's GPU (its UUID when torch reports one, so that
        a CUDA_VISIBLE_DEVICES remapping cannot point the sampler at another GPU)."""
        try:
            u = str(torch.cuda.get_device_properties(self.index).uuid)
            if u:
                return u if u.startswith("GPU-") else f"GPU-{u}"
        except Exception:
            pass
        return str(self.index)

    def start(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        for gid in dict.fromkeys([self._gpu_id(), str(self.index)]):
            try:
                self.f = open(self.path, "w")
                self.proc = subprocess.Popen(["nvidia-smi", f"--id={gid}", f"--query-gpu={q}",
                                              "--format=csv,noheader,nounits", "-lms", "200"],
                                             stdout=self.f, stderr=subprocess.DEVNULL)
            except Exception:
                self.proc = None
                return
            # do not start the timed region before the first sample is in (nvidia-smi can take
            # seconds to come up on a busy host)
            t0 = time.time()
            while time.time() - t0 < 15.0 and self.proc.poll() is None:
                try:
                    if os.path.getsize(self.path) > 0:
                        return
                except OSError:
                    pass
                time.sleep(0.05)
            if self.proc.poll() is None:
                return  # still running: samples may yet come
            self.f.close()  # this id was refused: try the next one

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    mx.append(float(parts[2]))
                except ValueError:
                    continue
                for n, v in zip(names, parts[5:9]):
                    if v.lower() == "active":
                        reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def reference_arm(args, rank):
    why = ("reference project (JAX/Flax/Optax/Orbax + Pallas-TPU kernels) is not installable offline: "
           "the reference source tree has no setup.py/pyproject.toml and jax is not in the image")
    try:
        sys.path.insert(0, os.path.join(HERE, "baseline", "_ref"))
        import jax  # noqa: F401
        import train_setup  # noqa: F401
    except Exception:
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": why}), flush=True)
        return


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        reference_arm(args, rank)
        return
    from datetime import timedelta

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    from atomic_ai_hybrid_b200 import get_preset, ops
    from atomic_ai_hybrid_b200.models import HybridMoEModel, count_params
    from atomic_ai_hybrid_b200.training.trainer import Trainer
    from atomic_ai_hybrid_b200.utils.counters import launch_counter

    ops.set_impl("cuda" if args.impl == "cuda" else "eager")
    over = {}
    if args.layers:
        over["num_layers"] = args.layers
    cfg = get_preset(args.model, **over)
    S, mb = args.seq_len, args.micro_batch
    tp = max(1, args.tp)
    if tp > 1:
        if world % tp:
            raise SystemExit("--tp must divide the number of GPUs")
        if args.ep > 1 and args.ep != tp:
            raise SystemExit("with --tp, --ep must equal --tp (experts split over the tensor-parallel group)")
        from atomic_ai_hybrid_b200.parallel.tp import init_tensor_parallel
        init_tensor_parallel(tp, dev, expert_parallel=args.ep > 1, max_rows=mb * S // tp, max_width=cfg.d_model)
    elif args.ep > 1:
        if args.ep != world:
            raise SystemExit("--ep must equal the number of GPUs")
        from atomic_ai_hybrid_b200.parallel.context import ParallelContext, set_parallel_context
        set_parallel_context(ParallelContext(dp_world=world, ep_world=world, ep_rank=rank))
    # the model draws every full tensor and keeps this rank's pieces: one seed for all ranks
    torch.manual_seed(1234)
    with torch.device(dev):
        model = HybridMoEModel(cfg, compute_dtype=torch.bfloat16, remat=args.remat)
    # N(0, 0.02) init of every matrix (benchmark spec), norms at 1, biases 0; replicated
    # matrices draw the same values on every rank, tensor- / expert-parallel pieces their own
    from atomic_ai_hybrid_b200.parallel.tp import shard_spec
    g_rep = torch.Generator(device=dev).manual_seed(1234)
    g_loc = torch.Generator(device=dev).manual_seed(1234 + 7919 * (rank + 1))
    with torch.no_grad():
        for n, p in model.named_parameters():
            if p.ndim >= 2 and "conv_w" not in n:
                local = shard_spec(p) is not None or getattr(p, "_ahb_ep_local", False)
                p.normal_(0.0, 0.02, generator=g_loc if local else g_rep)
    model = model.to(dev)
    nparams = count_params(model)
    use_graph = args.impl == "cuda" and not args.no_graph
    # the eager baseline keeps NCCL collectives; the CUDA path uses the peer-memory fused step
    trainer = Trainer(model, total_steps=1000, optimizer=args.optimizer, compute_dtype=torch.bfloat16, device=dev,
                      cuda_graph=use_graph, comm="nccl" if args.impl == "eager" else "auto",
                      ep_max_tokens=args.micro_batch * args.seq_len // tp if args.ep > 1 else 0,
                      expert_grad_bf16=args.expert_grad_bf16)
    trainer.opt.schedule.warmup = 1  # non-zero learning rate from the first step

    n_micro = max(1, args.seqs_per_gpu * tp // mb)
    seqs = n_micro * mb  # per data-parallel replica (one tensor-parallel group)
    gen = torch.Generator().manual_seed(17 + rank // tp)
    host_ids = torch.randint(0, cfg.vocab_size, (n_micro, mb, S + 1), generator=gen, dtype=torch.int32).pin_memory()
    dev_ids = host_ids.to(dev)

    def batches_dev():
        return [{"input_ids": dev_ids[i, :, :-1].long(), "labels": dev_ids[i, :, 1:].long()} for i in range(n_micro)]

    def barrier():
        if world > 1:
            dist.barrier()

    # warm-up
    for _ in range(args.warmup):
        trainer.train_step(batches_dev())
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()

    sampler = ClockSampler(local)
    sampler.start()
    launch_counter.reset()
    launch_counter.enable()
    trainer.phase_events = {} if args.impl == "cuda" else None
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(args.steps):
        out = trainer.train_step(batches_dev())
    ev1.record()
    torch.cuda.synchronize()
    phases = step_phases(trainer.phase_events, args.steps, world)
    trainer.phase_events = None
    launches = launch_counter.count
    if trainer.cuda_graph:  # kernels inside the replayed micro-step graph
        launches += trainer.graph_kernel_launches * n_micro * args.steps
    launch_counter.disable()
    barrier()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    ms = ev0.elapsed_time(ev1) / args.steps
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    tokens_step = seqs * S * (world // tp)
    value = tokens_step / (ms / 1e3)

    e2e = None
    if not args.no_e2e:
        # end to end through the public API: per step, H2D of the step's tokens from pinned
        # memory and D2H of the loss.
        h2d = 0
        torch.cuda.synchronize()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        w0 = time.perf_counter()
        e0.record()
        for _ in range(args.steps):
            ids = host_ids.to(dev, non_blocking=True)
            h2d += host_ids.numel() * host_ids.element_size()
            bs = [{"input_ids": ids[i, :, :-1].long(), "labels": ids[i, :, 1:].long()} for i in range(n_micro)]
            out = trainer.train_step(bs)
            _ = out["loss"].item()
        e1.record()
        torch.cuda.synchronize()
        wall = (time.perf_counter() - w0) / args.steps * 1e3
        t = torch.tensor([wall], device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        wall = float(t.item())
        e2e = {"value": tokens_step / (wall / 1e3), "unit": "tokens/s", "ms_per_step": wall,
               "h2d_bytes_per_step": h2d // args.steps, "d2h_bytes_per_step": 4,
               "loss": float(out["loss"].item())}

    scan = None
    if args.impl == "cuda" and not args.no_scan_ops and rank == 0:
        scan = scan_ops(dev)
    if rank == 0:
        line = {
            "metric": "train tokens/sec (box, max over ranks)",
            "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": (value / EAGER_BASELINE_TOKS if (world == 1 and args.model == "hybrid_1b"
                                                            and args.seq_len == 4096) else None),
            "dtype": "bf16", "data": "synthetic tokens, random-init weights",
            "impl": args.impl,
            "config": {"model": args.model, "global_batch": seqs * (world // tp), "seq_len": S,
                       "micro_batch": mb, "grad_accum": n_micro,
                       "parallelism": f"dp{world // tp}" + (f"+tp{tp}" if tp > 1 else "")
                       + (f"+ep{args.ep}" if args.ep > 1 else ""),
                       "sharding": "param/optimizer owner-sharded, bf16 weights resident",
                       "collectives": ("none" if world == 1 else
                                       "NVLink peer memory: reduce-scatter fused into the optimizer's first pass, "
                                       "all-gather fused into its update" if trainer.fused_comm else
                                       type(trainer.comm).__name__),
                       "optimizer": args.optimizer, "params_total": nparams["total"],
                       "num_layers": cfg.num_layers,
                       "peak_mem_gb": round(torch.cuda.max_memory_allocated(dev) / 1e9, 1) if dev.type == "cuda" else None,
                       "l2": "inputs larger than L2 (11+ GB of weights streamed per micro-step)"},
            "clocks": clocks, "e2e": e2e, "gpu_launches": launches,
            "phases_ms": phases,
        }
        if scan is not None:
            line["scan_ops"] = scan
        print(json.dumps(line), flush=True)
    shutdown(trainer, world)


def step_phases(events, steps: int, world: int):
    """Per-step device time of the training step's phases over the timed steps, max over
    ranks: the micro-steps (forward, backward, accumulation), the barrier before the optimizer,
    the optimizer (with the NVLink peer-memory reduce-scatter fused into its first pass and the
    all-gather into its update), and the barrier after it."""
    if not events or len(events.get("micro", [])) != steps:
        return None
    spans = {"micro_steps": ("micro", "apply"), "begin_barrier": ("apply", "optimizer"),
             "optimizer_fused_comm": ("optimizer", "end_barrier"), "end_barrier": ("end_barrier", "done")}
    vals = []
    for a, b in spans.values():
        vals.append(sum(x.elapsed_time(y) for x, y in zip(events[a], events[b])) / steps)
    t = torch.tensor(vals, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return {k: round(float(v), 3) for k, v in zip(spans, t.tolist())}


def scan_ops(dev):
    """The scan operators at the benchmark's operator configuration (GDN-2 B 8, T 4096, H 16,
    D 128; Mamba2 SSD B 8, T 4096, H 32, P 64, N 128), forward + backward, bf16, CUDA events with
    an L2 flush between iterations; TFLOP/s of the chunked algorithm's matmul FLOPs and the
    fraction of the HBM roofline (minimum input / output bytes over the measured copy bandwidth)."""
    from atomic_ai_hybrid_b200.utils import opbench
    peaks = {}
    try:
        with open(os.path.join(HERE, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except OSError:
        pass
    hbm = float(peaks.get("hbm_gbs", 6650.0))
    flush = torch.empty(64 << 20, dtype=torch.float32, device=dev)
    out = {}
    for name, fn, H in (("gdn2", opbench.bench_gdn, 16), ("ssd", opbench.bench_ssd, 32)):
        r = fn(8, 4096, H, 2, 5, flush)
        out[name] = {"ms": round(r["ms"], 3), "tflops": round(r["tflops"], 1),
                     "hbm_roofline_fraction": round(r["min_io_gb_s"] / hbm, 3), "shape": f"B8 T4096 H{H}"}
    del flush
    torch.cuda.empty_cache()
    return out


def shutdown(trainer, world: int, deadline_s: float = 120.0) -> None:
    """Release the CUDA graph (it may hold NCCL collectives) and tear the process
    group down; if teardown stalls past the deadline, exit the process directly."""
    import gc
    import threading

    def force_exit():
        sys.stdout.flush()
        sys.stderr.flush()
        os._exit(0)

    timer = threading.Timer(deadline_s, force_exit)
    timer.daemon = True
    timer.start()
    trainer.close()
    gc.collect()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    timer.cancel()


if __name__ == "__main__":
    main()
