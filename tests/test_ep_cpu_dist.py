"""Expert parallelism through the torch.distributed all-to-all (gloo ranks on the CPU):
the model with its routed experts split over 2, 4 or 8 ranks gives the single-rank loss and
gradients, and trains like it."""
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from atomic_ai_hybrid_b200 import get_preset
from atomic_ai_hybrid_b200.models import HybridMoEModel
from atomic_ai_hybrid_b200.parallel.context import ParallelContext, set_parallel_context
from atomic_ai_hybrid_b200.training.loss import compute_loss
from _dist import collect, free_port as _port, threads_per_rank




def _cfg(world=2):
    return get_preset("tiny", num_layers=2, layer_types=("mamba2", "gdn2"), vocab_size=512, d_model=128,
                      n_heads=2, n_heads_ssm=2, d_ff=128, n_routed_experts=max(4, world), top_k=2, d_state=32)


def _worker(rank, world, port, q, ep=None):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.set_num_threads(threads_per_rank(world))
    try:
        cfg = _cfg(world)
        # every rank: the single-rank model on the whole global batch (2 sequences per rank)
        set_parallel_context(ParallelContext())
        torch.manual_seed(0)
        full = HybridMoEModel(cfg, compute_dtype=torch.float32)
        ids = torch.randint(0, cfg.vocab_size, (2 * world, 65), generator=torch.Generator().manual_seed(5))
        full.zero_grad()
        lf, _ = compute_loss(full, {"input_ids": ids[:, :-1], "labels": ids[:, 1:]})
        lf.backward()
        gf = {n: p.grad.clone() for n, p in full.named_parameters() if p.grad is not None}
        # experts split over the ranks, each rank on its own 2 sequences (data parallel)
        from atomic_ai_hybrid_b200.parallel.ep import init_expert_parallel
        ctx = init_expert_parallel(ep or world)
        torch.manual_seed(0)
        m = HybridMoEModel(cfg, compute_dtype=torch.float32)
        mine = ids[2 * rank:2 * rank + 2]
        m.zero_grad()
        loss, _ = compute_loss(m, {"input_ids": mine[:, :-1], "labels": mine[:, 1:]})
        loss.backward()
        lt = loss.detach().clone()
        dist.all_reduce(lt)
        res = {"loss": float((lt / world - lf).abs() / lf.abs())}
        worst, which = 0.0, None
        ep = ep or world
        El = cfg.e_routed // ep
        er = rank % ep
        for n, p in m.named_parameters():
            if p.grad is None:
                continue
            g = p.grad.clone()
            if getattr(p, "_ahb_ep_local", False):
                if ctx.local_group is not None:  # the replicas holding the same experts
                    dist.all_reduce(g, group=ctx.local_group)
                ref = gf[n][er * El:(er + 1) * El]
                got = g / world            # summed over every rank's tokens; the reference is their mean
            else:
                dist.all_reduce(g)
                got, ref = g / world, gf[n]
            e = float((got - ref).abs().max() / ref.abs().max().clamp_min(1e-6))
            if e > worst:
                worst, which = e, n
        res["grad"], res["worst"] = worst, which
        q.put((rank, res))
    finally:
        set_parallel_context(ParallelContext())
        dist.destroy_process_group()


@pytest.mark.parametrize("world,ep", [(2, 2), (4, 4), (8, 8), (4, 2)])
def test_ep_collective_matches_single_rank(world, ep):
    """2, 4 and 8 ranks (8 routed experts at 8 ranks: one per rank); and two data-parallel
    replicas of a 2-rank expert-parallel group."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, ep)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(collect(procs, q, len(procs), 300))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(world):
        assert res[r]["loss"] < 1e-5, res
        assert res[r]["grad"] < 1e-3, res
