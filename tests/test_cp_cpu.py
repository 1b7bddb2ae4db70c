"""Context parallelism on CPU ranks (gloo): each rank holds one segment of every sequence;
the scans pass their states across the segment boundaries, the convolutions a halo, MLA
the latent of every position.  The loss and gradients equal the single-rank model's."""
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




def _cfg(kind):
    if kind == "interleaved":
        return get_preset("tiny", num_layers=2, layer_types=("mamba2", "gdn2"), vocab_size=512, d_model=128,
                          n_heads=2, n_heads_ssm=2, d_ff=128, n_routed_experts=4, d_state=32)
    return get_preset("reference_tiny", dropout_rate=0.0, router_noise_std=0.0)


def _worker(rank, world, port, kind, q, cp=None):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.set_num_threads(threads_per_rank(world))
    try:
        from atomic_ai_hybrid_b200.parallel.cp import init_context_parallel
        cfg = _cfg(kind)
        set_parallel_context(ParallelContext())
        torch.manual_seed(0)
        full = HybridMoEModel(cfg, compute_dtype=torch.float32)
        cp = cp or world
        reps = world // cp  # data-parallel replicas of the context-parallel group
        ids = torch.randint(0, cfg.vocab_size, (2 * reps, 64 * cp + 1), generator=torch.Generator().manual_seed(7))
        lf, _ = compute_loss(full, {"input_ids": ids[:, :-1], "labels": ids[:, 1:]})
        d = rank // cp
        batch = {"input_ids": ids[2 * d:2 * d + 2, :-1], "labels": ids[2 * d:2 * d + 2, 1:]}
        lf.backward()
        gf = {n: p.grad.clone() for n, p in full.named_parameters() if p.grad is not None}
        init_context_parallel(cp_size=cp)
        m = HybridMoEModel(cfg, compute_dtype=torch.float32)
        m.load_state_dict(full.state_dict())
        loss, _ = compute_loss(m, batch)
        loss.backward()
        lt = loss.detach().clone()
        dist.all_reduce(lt)
        res = {"loss": float((lt / world - lf).abs() / lf.abs())}
        worst, which = 0.0, None
        for n, p in m.named_parameters():
            if p.grad is None:
                continue
            g = p.grad.clone()
            dist.all_reduce(g)
            e = float((g / world - gf[n]).abs().max() / gf[n].abs().max().clamp_min(1e-6))
            if os.environ.get("CP_DEBUG") and rank == 0 and e > 1e-3:
                print(f"CPDBG {n} {e:.3e}", flush=True)
            if e > worst:
                worst, which = e, n
        res["grad"], res["worst"] = worst, which
        q.put((rank, res))
    finally:
        set_parallel_context(ParallelContext())
        dist.destroy_process_group()


@pytest.mark.parametrize("kind,world,cp", [("interleaved", 2, 2), ("interleaved", 4, 4), ("blockdar", 2, 2),
                                           ("interleaved", 4, 2)])
def test_cp_matches_single_rank(kind, world, cp):
    """``cp < world``: two data-parallel replicas of a 2-rank context-parallel group, each
    with its own sequences; the reference model sees both replicas' sequences."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, kind, q, cp)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(collect(procs, q, len(procs), 600))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(world):
        assert res[r]["loss"] < 1e-5, res
        # per-head decay scalars sum over every token and channel: fp32 reduction order
        assert res[r]["grad"] < 1e-3, res
