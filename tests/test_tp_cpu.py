"""Tensor + sequence parallelism on CPU ranks (gloo): a model whose mixer heads are
split over 2 ranks (token rows split between the mixers) must give the loss and
gradients of the single-rank model with the same weights, and training with the
tensor-parallel trainer must follow single-rank training."""
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




def _cfg(kind, world=2):
    if kind == "interleaved":
        return get_preset("tiny", num_layers=2, layer_types=("mamba2", "gdn2"), vocab_size=512, d_model=128,
                          n_heads=max(2, world), n_heads_ssm=4, d_ff=128, n_routed_experts=4, d_state=32)
    return get_preset("reference_tiny", dropout_rate=0.0, router_noise_std=0.0)


def _loss_grads(model, ids):
    model.zero_grad(set_to_none=True)
    loss, _ = compute_loss(model, {"input_ids": ids[:, :-1], "labels": ids[:, 1:]}, deterministic=False)
    loss.backward()
    return loss.detach(), {n: (p.grad.clone() if p.grad is not None else torch.zeros_like(p))
                           for n, p in model.named_parameters()}


def _parity(rank, world, port, kind, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.set_num_threads(threads_per_rank(world))
    try:
        from atomic_ai_hybrid_b200.parallel.tp import init_tensor_parallel, load_full_state, shard_spec, shard_tensor
        cfg = _cfg(kind, world)
        set_parallel_context(ParallelContext())
        torch.manual_seed(0)
        full = HybridMoEModel(cfg, compute_dtype=torch.float32)
        g = torch.Generator().manual_seed(3)
        ids = torch.randint(0, cfg.vocab_size, (2, 129), generator=g)
        loss_f, grads_f = _loss_grads(full, ids)

        init_tensor_parallel(world, torch.device("cpu"))
        torch.manual_seed(0)
        tpm = HybridMoEModel(cfg, compute_dtype=torch.float32)
        # built from the same seed, the split model already holds the pieces of the full one
        fsd = full.state_dict()
        init_diff = 0.0
        for n, p in tpm.named_parameters():
            spec = shard_spec(p)
            ref = shard_tensor(fsd[n], spec[0], spec[1], world, rank) if spec is not None else fsd[n]
            init_diff = max(init_diff, float((p.detach() - ref).abs().max()))
        load_full_state(tpm, fsd)
        loss_t, grads_t = _loss_grads(tpm, ids)
        lt = loss_t.clone()
        dist.all_reduce(lt)
        errs = {"loss": float((lt / world - loss_f).abs() / loss_f.abs()), "init": init_diff}
        worst = 0.0
        for n, p in tpm.named_parameters():
            gt = grads_t[n]
            spec = shard_spec(p)
            if spec is not None:
                ref = shard_tensor(grads_f[n], spec[0], spec[1], world, rank)
                got = gt / world
            else:
                got = gt.clone()
                dist.all_reduce(got)
                got = got / world
                ref = grads_f[n]
            den = ref.abs().max().clamp_min(1e-6)
            e = float((got - ref).abs().max() / den)
            if e > worst:
                worst, errs["worst"] = e, n
        errs["grad"] = worst
        q.put((rank, errs))
    finally:
        set_parallel_context(ParallelContext())
        dist.destroy_process_group()


@pytest.mark.parametrize("kind,world", [("interleaved", 2), ("blockdar", 2), ("interleaved", 4)])
def test_tp_forward_backward_matches_single_rank(kind, world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_parity, args=(r, world, port, kind, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = collect(procs, q, len(procs))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, errs in res:
        assert errs["init"] == 0.0, (rank, errs)
        assert errs["loss"] < 1e-5, (rank, errs)
        # per-head decay gradients sum over every token and channel: fp32 reduction order
        assert errs["grad"] < 1e-3, (rank, errs)


def _train(rank, world, port, steps, q, optimizer="adamw"):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    if world > 1:
        dist.init_process_group("gloo", rank=rank, world_size=world)
        torch.set_num_threads(threads_per_rank(world))
    try:
        from atomic_ai_hybrid_b200.parallel.tp import init_tensor_parallel, load_full_state, unshard_tensors, shard_spec
        from atomic_ai_hybrid_b200.training.trainer import Trainer
        cfg = _cfg("interleaved")
        set_parallel_context(ParallelContext())
        torch.manual_seed(0)
        full = HybridMoEModel(cfg, compute_dtype=torch.float32)
        init = {n: p.detach().clone() for n, p in full.named_parameters()}
        if world > 1:
            init_tensor_parallel(world, torch.device("cpu"))
            m = HybridMoEModel(cfg, compute_dtype=torch.float32)
            load_full_state(m, full.state_dict())
        else:
            m = full
        tr = Trainer(m, total_steps=50, optimizer=optimizer, compute_dtype=torch.float32, device=torch.device("cpu"))
        tr.opt.schedule.warmup = 1
        g = torch.Generator().manual_seed(9)
        ids = torch.randint(0, cfg.vocab_size, (2, 129), generator=g)
        hist = []
        for _ in range(steps):
            out = tr.train_step([{"input_ids": ids[:, :-1], "labels": ids[:, 1:]}])
            loss = out["loss"].clone()
            if world > 1:
                dist.all_reduce(loss)
            hist.append((float(loss) / world, float(out["global_norm"])))
        res = {}
        for n, p in m.named_parameters():
            t = p.detach().float().clone()
            spec = shard_spec(p)
            if spec is not None and world > 1:
                parts = [torch.zeros_like(t) for _ in range(world)]
                dist.all_gather(parts, t)
                t = unshard_tensors(parts, spec[0], spec[1])
            res[n] = (t - init[n]).numpy()
        if rank == 0:
            q.put((hist, res))
        tr.close()
    finally:
        set_parallel_context(ParallelContext())
        if world > 1:
            dist.destroy_process_group()


@pytest.mark.parametrize("optimizer", ["adamw", "hybrid"])
def test_tp2_training_follows_single_rank(optimizer):
    """Losses and global gradient norms per step match; every parameter (split
    pieces included) moves, and by the same amount up to Adam's sign sensitivity on
    near-zero gradients (bounded by the learning rate).  With the hybrid optimizer the
    Muon matrices split over the ranks are orthogonalised whole."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    steps = 3
    p1 = ctx.Process(target=_train, args=(0, 1, _port(), steps, q, optimizer))
    p1.start()
    (ref_hist, ref), = collect([p1], q, 1)
    p1.join(timeout=60)
    port = _port()
    procs = [ctx.Process(target=_train, args=(r, 2, port, steps, q, optimizer)) for r in range(2)]
    for p in procs:
        p.start()
    (hist, got), = collect(procs, q, 1)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for (l0, n0), (l1, n1) in zip(ref_hist, hist):
        assert abs(l1 - l0) <= 1e-5 * abs(l0), (ref_hist, hist)
        assert abs(n1 - n0) <= 1e-4 * abs(n0), (ref_hist, hist)
    for n, r in ref.items():
        r, t = torch.from_numpy(r), torch.from_numpy(got[n])
        if r.abs().max() > 0:
            assert t.abs().max() > 0, f"{n} did not move"
        assert (t - r).abs().max() <= 2 * 6e-4 * steps, n


def test_tp_checkpoint_pieces_reassemble_for_any_world():
    from atomic_ai_hybrid_b200.ckpt.manager import _lookup_tp
    from atomic_ai_hybrid_b200.parallel.tp import shard_tensor
    full = torch.arange(6 * 16, dtype=torch.float32).view(6, 16)
    for dim, parts in ((1, 1), (1, 2), (0, 1)):
        pieces = {f"w#tp[{r}/2]": shard_tensor(full, dim, parts, 2, r) for r in range(2)}
        for world in (1, 2):
            for rank in range(world):
                got = _lookup_tp(pieces, "w", (dim, parts, rank, world))
                assert torch.equal(got, shard_tensor(full, dim, parts, world, rank))
        assert torch.equal(_lookup_tp({"w": full}, "w", (dim, parts, 1, 2)), shard_tensor(full, dim, parts, 2, 1))
    del pieces["w#tp[1/2]"]
    assert _lookup_tp(pieces, "w", (0, 1, 0, 1)) is None


def _ckpt(rank, world, port, root, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.set_num_threads(threads_per_rank(world))
    try:
        from atomic_ai_hybrid_b200.ckpt.manager import CheckpointManager
        from atomic_ai_hybrid_b200.parallel.tp import init_tensor_parallel, load_full_state, shard_spec, unshard_tensors
        from atomic_ai_hybrid_b200.training.trainer import Trainer
        cfg = _cfg("interleaved")
        solo = dist.new_group([0])
        set_parallel_context(ParallelContext())
        torch.manual_seed(0)
        full = HybridMoEModel(cfg, compute_dtype=torch.float32)
        init_tensor_parallel(world, torch.device("cpu"))
        m = HybridMoEModel(cfg, compute_dtype=torch.float32)
        load_full_state(m, full.state_dict())
        tr = Trainer(m, total_steps=10, optimizer="adamw", compute_dtype=torch.float32, device=torch.device("cpu"))
        tr.opt.schedule.warmup = 1
        ids = torch.randint(0, cfg.vocab_size, (2, 129), generator=torch.Generator().manual_seed(4))
        tr.train_step([{"input_ids": ids[:, :-1], "labels": ids[:, 1:]}])
        ck = CheckpointManager(root, rank=rank, world=world)
        ck.save(1, tr, asynchronous=False)
        dist.barrier()
        # the full (unsplit) weights after the step
        ref = {}
        for n, p in m.named_parameters():
            t = p.detach().clone()
            spec = shard_spec(p)
            if spec is not None:
                parts = [torch.zeros_like(t) for _ in range(world)]
                dist.all_gather(parts, t)
                t = unshard_tensors(parts, spec[0], spec[1])
            ref[n] = t
        # restore into a fresh tensor-parallel model
        m2 = HybridMoEModel(cfg, compute_dtype=torch.float32)
        tr2 = Trainer(m2, total_steps=10, optimizer="adamw", compute_dtype=torch.float32, device=torch.device("cpu"))
        meta = CheckpointManager(root, rank=rank, world=world).restore(1, tr2)
        def err(n, a, b):
            # routed experts are stored in bf16 (the reference's dtype): within bf16 rounding of
            # the largest element; everything else bit-exact
            d = float((a.detach() - b.detach()).abs().max())
            if "routed_w" in n:
                return 0.0 if d <= float(b.abs().max()) * 2 ** -8 else d
            return d

        b_of = dict(m.named_parameters())
        res = {"tp_restore": max(err(n, p, b_of[n]) for n, p in m2.named_parameters()), "fresh": len(meta["fresh"])}
        dist.barrier()
        if rank == 0:
            # and into a single-rank model: every piece reassembled
            set_parallel_context(ParallelContext())
            m1 = HybridMoEModel(cfg, compute_dtype=torch.float32)
            tr1 = Trainer(m1, total_steps=10, optimizer="adamw", compute_dtype=torch.float32,
                          device=torch.device("cpu"), group=solo)
            meta1 = CheckpointManager(root, rank=0, world=1).restore(1, tr1)
            res["single_restore"] = max(err(n, p, ref[n]) for n, p in m1.named_parameters())
            res["single_fresh"] = len(meta1["fresh"])
        q.put((rank, res))
        dist.barrier()
    finally:
        set_parallel_context(ParallelContext())
        dist.destroy_process_group()


def test_tp_checkpoint_restores_into_tp_and_single_rank(tmp_path):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_ckpt, args=(r, 2, port, str(tmp_path), q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(collect(procs, q, len(procs), 300))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(2):
        assert res[r]["fresh"] == 0 and res[r]["tp_restore"] == 0.0, res
    assert res[0]["single_fresh"] == 0 and res[0]["single_restore"] == 0.0, res
