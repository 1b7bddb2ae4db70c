"""Pipeline parallelism on CPU ranks (gloo): two stages of the interleaved stack (the
first with the embedding, the last with the final norm and the tied LM head) train like
the single-rank model -- same losses and gradient norms per step, same weights after."""
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from atomic_ai_hybrid_b200 import get_preset
from atomic_ai_hybrid_b200.models import HybridMoEModel
from atomic_ai_hybrid_b200.parallel.context import ParallelContext, set_parallel_context


from _dist import collect, free_port as _port, threads_per_rank


def _cfg(layers):
    return get_preset("tiny", num_layers=layers, layer_types=("mamba2", "gdn2", "gdn2", "mamba2")[:layers],
                      vocab_size=512, d_model=128, n_heads=2, n_heads_ssm=2, d_ff=128, n_routed_experts=4,
                      d_state=32)


def _run(rank, world, port, steps, layers, q, schedule="1f1b", dp=1):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    if world > 1:
        dist.init_process_group("gloo", rank=rank, world_size=world)
        torch.set_num_threads(threads_per_rank(world))
    try:
        from atomic_ai_hybrid_b200.training.trainer import Trainer
        from atomic_ai_hybrid_b200.parallel.pp import PipelineTrainer
        set_parallel_context(ParallelContext())
        cfg = _cfg(layers)
        torch.manual_seed(0)
        m = HybridMoEModel(cfg, compute_dtype=torch.float32)
        if world > 1:
            tr = PipelineTrainer(m, total_steps=50, optimizer="adamw", device=torch.device("cpu"),
                                 schedule=schedule, data_parallel=dp)
        else:
            tr = Trainer(m, total_steps=50, optimizer="adamw", compute_dtype=torch.float32,
                         device=torch.device("cpu"))
        tr.opt.schedule.warmup = 1
        g = torch.Generator().manual_seed(9)
        ids = torch.randint(0, cfg.vocab_size, (4, 129), generator=g)
        micro = [{"input_ids": ids[i:i + 1, :-1], "labels": ids[i:i + 1, 1:]} for i in range(4)]
        if world > 1 and dp > 1:  # replica d takes its share of the micro-batches
            per = len(micro) // dp
            d = rank // (world // dp)
            micro = micro[d * per:(d + 1) * per]
        hist = []
        for _ in range(steps):
            out = tr.train_step(micro)
            loss = out["loss"].clone()
            if world > 1 and dp > 1:  # the replicas' mean is the single-rank loss
                dist.all_reduce(loss)
                loss /= world
            hist.append((float(loss), float(out["global_norm"])))
        params = {n: p.detach().clone().numpy() for n, p in m.named_parameters()}
        peak = 0
        if world > 1:
            held = {n for n, _ in tr.part.named_parameters()}
            params = {n: v for n, v in params.items() if n in held}
            peak = tr.peak_live
        q.put((rank, hist, params, peak))
    finally:
        if world > 1:
            dist.destroy_process_group()


def _reference(steps, layers):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p1 = ctx.Process(target=_run, args=(0, 1, _port(), steps, layers, q))
    p1.start()
    (_, ref_hist, ref, _), = collect([p1], q, 1)
    p1.join(timeout=60)
    return ref_hist, ref


def _pipeline(world, steps, layers, schedule, dp=1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_run, args=(r, world, port, steps, layers, q, schedule, dp)) for r in range(world)]
    for p in procs:
        p.start()
    got = collect(procs, q, len(procs))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return sorted(got, key=lambda t: t[0])


def _check(ref_hist, ref, got, steps):
    for _, hist, params, _ in got:
        for (l0, n0), (l1, n1) in zip(ref_hist, hist):
            assert abs(l1 - l0) <= 1e-5 * abs(l0), (ref_hist, hist)
            assert abs(n1 - n0) <= 1e-4 * abs(n0), (ref_hist, hist)
        for n, v in params.items():
            r, t = torch.from_numpy(ref[n]), torch.from_numpy(v)
            assert (t - r).abs().max() <= 2 * 6e-4 * steps, n
    held = set().union(*(set(p) for _, _, p, _ in got))
    assert held == set(ref), set(ref) ^ held


@pytest.mark.parametrize("stages,layers,schedule", [(2, 2, "1f1b"), (2, 3, "gpipe"), (3, 3, "1f1b")])
def test_pipeline_training_follows_single_rank(stages, layers, schedule):
    """Even and uneven layer splits, both schedules: the loss, the gradient norm and the
    weights after three steps match one rank running every micro-batch."""
    steps = 3
    ref_hist, ref = _reference(steps, layers)
    got = _pipeline(stages, steps, layers, schedule)
    _check(ref_hist, ref, got, steps)
    peaks = [g[3] for g in got]
    if schedule == "1f1b":  # stage s keeps at most S - s micro-batches' activations
        assert peaks == [min(stages - s, 4) for s in range(stages)], peaks
    else:
        assert peaks == [4] * stages, peaks


def test_pipeline_with_data_parallel_replicas():
    """A 2 x 2 mesh (two replicas of a two-stage pipeline, each stage's store sharded over
    its two replicas) trains like one rank running both replicas' micro-batches."""
    steps = 2
    ref_hist, ref = _reference(steps, 2)
    got = _pipeline(4, steps, 2, "1f1b", dp=2)
    _check(ref_hist, ref, got, steps)


def _ckpt(rank, world, port, root, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.set_num_threads(threads_per_rank(world))
    try:
        from atomic_ai_hybrid_b200.ckpt.manager import CheckpointManager
        from atomic_ai_hybrid_b200.parallel.pp import PipelineTrainer
        from atomic_ai_hybrid_b200.training.trainer import Trainer
        set_parallel_context(ParallelContext())
        cfg = _cfg(3)
        solo = dist.new_group([0])
        torch.manual_seed(0)
        m = HybridMoEModel(cfg, compute_dtype=torch.float32)
        tr = PipelineTrainer(m, total_steps=50, optimizer="adamw", device=torch.device("cpu"))
        tr.opt.schedule.warmup = 1
        ids = torch.randint(0, cfg.vocab_size, (2, 129), generator=torch.Generator().manual_seed(2))
        tr.train_step([{"input_ids": ids[:, :-1], "labels": ids[:, 1:]}])
        CheckpointManager(root, rank=rank, world=world).save(1, tr, asynchronous=False)
        dist.barrier()
        held = {n: p.detach().clone() for n, p in tr.part.named_parameters()}
        if rank == 0:
            torch.manual_seed(5)
            m1 = HybridMoEModel(cfg, compute_dtype=torch.float32)
            t1 = Trainer(m1, total_steps=50, optimizer="adamw", compute_dtype=torch.float32,
                         device=torch.device("cpu"), group=solo)
            meta = CheckpointManager(root, rank=0, world=1).restore(1, t1)
            q.put(("meta", len(meta["fresh"]), {n: p.detach().clone().numpy() for n, p in m1.named_parameters()}))
        q.put(("held", rank, {n: v.numpy() for n, v in held.items()}))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_pp_checkpoint_restores_single_rank(tmp_path):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_ckpt, args=(r, 2, port, str(tmp_path), q)) for r in range(2)]
    for p in procs:
        p.start()
    msgs = collect(procs, q, 3)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    fresh, restored = next((m[1], m[2]) for m in msgs if m[0] == "meta")
    assert fresh == 0
    for kind, _, held in (m for m in msgs if m[0] == "held"):
        for n, v in held.items():
            ref = torch.from_numpy(restored[n])
            t = torch.from_numpy(v)
            if "routed_w" in n:  # bf16 in the files, as in the reference
                t = t.to(torch.bfloat16).float()
            assert torch.equal(ref, t), n
