"""Sharded data parallelism on CPU ranks (gloo): the owner-sharded optimizer with
reduce-scatter / all-gather must reproduce single-process training on the same
global batch."""
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from atomic_ai_hybrid_b200 import get_preset
from atomic_ai_hybrid_b200.models import HybridMoEModel
from atomic_ai_hybrid_b200.training.trainer import Trainer
from _dist import collect, free_port as _port, threads_per_rank




def _cfg():
    return get_preset("tiny", num_layers=2, layer_types=("mamba2", "gdn2"), vocab_size=512, d_model=128,
                      n_heads=2, n_heads_ssm=2, d_ff=128, n_routed_experts=4, d_state=32)


def _batches(cfg, world):
    g = torch.Generator().manual_seed(5)
    ids = torch.randint(0, cfg.vocab_size, (2 * world, 65), generator=g)
    return ids


def _run(rank, world, port, out_path, steps):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    if world > 1:
        dist.init_process_group("gloo", rank=rank, world_size=world)
        torch.set_num_threads(threads_per_rank(world))
    cfg = _cfg()
    torch.manual_seed(0)
    m = HybridMoEModel(cfg, compute_dtype=torch.float32)
    tr = Trainer(m, total_steps=50, optimizer="hybrid", compute_dtype=torch.float32, device=torch.device("cpu"))
    tr.opt.schedule.warmup = 1
    ids = _batches(cfg, 4)  # 8 sequences: 1, 2 or 4 per rank at world 8, 4 or 2
    per = ids.shape[0] // world
    mine = ids[rank * per:(rank + 1) * per]
    for _ in range(steps):
        tr.train_step([{"input_ids": mine[:, :-1], "labels": mine[:, 1:]}])
    sd = tr.store.full_state_dict()
    if world > 1:
        # owners hold the exact fp32 masters: gather them
        full = {}
        for s in tr.store.segs:
            t = sd[s.name] if s.owner == rank else torch.zeros(s.shape)
            dist.broadcast(t, src=s.owner)
            full[s.name] = t
        sd = full
        dist.barrier()
    if rank == 0:
        torch.save(sd, out_path)
    if world > 1:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sharded_training_matches_single_process(tmp_path, world):
    steps = 3
    p1 = str(tmp_path / "one.pt")
    _run(0, 1, _port(), p1, steps)
    p2 = str(tmp_path / f"w{world}.pt")
    mp.spawn(_run, args=(world, _port(), p2, steps), nprocs=world, join=True)
    a, b = torch.load(p1), torch.load(p2)
    assert a.keys() == b.keys()
    # the MoE router noise is disabled in this config; every update is deterministic
    for k in a:
        torch.testing.assert_close(b[k], a[k], rtol=2e-4, atol=2e-5, msg=k)
