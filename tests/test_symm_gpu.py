"""NVLink peer-memory data parallelism: barrier, peer reduce / copy-out kernels,
the optimizer's fused reduce + push, and (with two GPUs) the whole fused step
against the NCCL step.

Single-GPU tests emulate the peers with several local buffers in the pointer
tables: the kernels only see device pointers.  The timeout test makes a barrier
wait on a flag that nothing sets and checks the error word it reports.
"""
import os
import tempfile
from datetime import timedelta

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ext():
    from atomic_ai_hybrid_b200.ops._ext import ext
    return ext()


def _tiny_cfg():
    from atomic_ai_hybrid_b200 import get_preset
    return get_preset("hybrid_1b", d_model=256, n_heads=2, n_heads_ssm=4, num_layers=2, d_ff=256,
                      n_routed_experts=8, top_k=2, vocab_size=1024, d_state=128)


def test_barrier_timeout_reports_error():
    E = _ext()
    dev = torch.device("cuda", 0)
    pad = E.ipc_alloc(256)
    try:
        err = torch.zeros(1, dtype=torch.int32, device=dev)
        # one rank: its own arrival satisfies the barrier
        E.symm_barrier(torch.tensor([pad], dtype=torch.int64, device=dev), 0, 1, err, 1.0)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        # two "ranks" on one pad: slot 1 is never written, so the wait must give up
        E.symm_barrier(torch.tensor([pad, pad], dtype=torch.int64, device=dev), 0, 2, err, 0.3)
        torch.cuda.synchronize()
        assert int(err.item()) == 101
    finally:
        E.ipc_free(pad)


def test_peer_reduce_and_copy_out():
    E = _ext()
    dev = torch.device("cuda", 0)
    n, W = 4096, 3
    bufs = [torch.randn(n, device=dev) for _ in range(W)]
    table = torch.tensor([b.data_ptr() for b in bufs], dtype=torch.int64, device=dev)
    lo, cnt = 1024, 2048
    out = torch.empty(cnt, device=dev)
    E.reduce_scatter_f32(table, lo, out)
    torch.testing.assert_close(out, sum(b[lo:lo + cnt] for b in bufs), rtol=1e-6, atol=1e-6)
    # in place into the first buffer's slice
    ref = sum(b[lo:lo + cnt] for b in bufs).clone()
    E.reduce_scatter_f32(table, lo, bufs[0][lo:lo + cnt])
    torch.testing.assert_close(bufs[0][lo:lo + cnt], ref, rtol=1e-6, atol=1e-6)
    # copy-out of a bf16 slice to every buffer
    cb = [torch.zeros(n, dtype=torch.bfloat16, device=dev) for _ in range(W)]
    ct = torch.tensor([c.data_ptr() for c in cb], dtype=torch.int64, device=dev)
    src = torch.randn(512, device=dev).to(torch.bfloat16)
    E.copy_out(src, ct, 256 * 2)
    torch.cuda.synchronize()
    for c in cb:
        assert torch.equal(c[256:768], src)
        assert not c[:256].any() and not c[768:].any()


def test_fused_optimizer_peer_tables():
    """prepare sums the slice over the gradient table; apply writes every compute buffer."""
    from atomic_ai_hybrid_b200 import ops
    from atomic_ai_hybrid_b200.models import HybridMoEModel
    from atomic_ai_hybrid_b200.optim import FlatParamStore, HybridOptimizer, grad_scale_of, label_of
    ops.set_impl("cuda")
    cfg = _tiny_cfg()
    dev = torch.device("cuda", 0)
    stores, opts = [], []
    for _ in range(2):
        torch.manual_seed(0)
        m = HybridMoEModel(cfg, compute_dtype=torch.bfloat16).to(dev)
        st = FlatParamStore(m, label_of, grad_scale_of, compute_dtype=torch.bfloat16, device=dev)
        opt = HybridOptimizer(st, total_steps=100)
        opt.schedule.warmup = 1
        stores.append(st)
        opts.append(opt)
    g = torch.Generator(device=dev).manual_seed(3)
    other_g = torch.zeros_like(stores[1].grad)
    other_c = torch.zeros_like(stores[1].compute)
    opts[1].peers = (torch.tensor([stores[1].grad.data_ptr(), other_g.data_ptr()], dtype=torch.int64, device=dev),
                     torch.tensor([stores[1].compute.data_ptr(), other_c.data_ptr()], dtype=torch.int64, device=dev))
    for _ in range(2):
        g0 = torch.randn(stores[0].grad.shape, device=dev, generator=g) * 0.01
        g1 = torch.randn(stores[0].grad.shape, device=dev, generator=g) * 0.01
        stores[0].grad.copy_(g0 + g1)
        stores[1].grad.copy_(g0)
        other_g.copy_(g1)
        opts[0].step(2)
        opts[1].step(2)
    torch.cuda.synchronize()
    torch.testing.assert_close(stores[1].master, stores[0].master, rtol=1e-6, atol=1e-7)
    # bitwise (fp32 tensors live as pairs of 16-bit units, which may read as NaN in bf16)
    assert torch.equal(stores[1].compute.view(torch.int16), stores[0].compute.view(torch.int16))
    assert torch.equal(other_c.view(torch.int16), stores[0].compute.view(torch.int16))


# ---------------------------------------------------------------- two ranks

def _worker(rank, world, port, outdir):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    from atomic_ai_hybrid_b200 import ops
    from atomic_ai_hybrid_b200.models import HybridMoEModel
    from atomic_ai_hybrid_b200.training.trainer import Trainer
    res = {}
    cfg = _tiny_cfg()
    for impl in ("cuda", "eager"):
        ops.set_impl(impl)
        trs = {}
        for kind in ("symm", "nccl"):
            torch.manual_seed(0)
            m = HybridMoEModel(cfg, compute_dtype=torch.bfloat16).to(dev)
            tr = Trainer(m, total_steps=100, optimizer="hybrid", device=dev, comm=kind)
            tr.opt.schedule.warmup = 1
            trs[kind] = tr
        res[f"{impl}_fused"] = trs["symm"].fused_comm
        g = torch.Generator(device=dev).manual_seed(7 + rank)
        for _ in range(2):
            grad = torch.randn(trs["nccl"].store.grad.shape, device=dev, generator=g) * 0.01
            for tr in trs.values():
                tr.store.grad.copy_(grad)
                tr.apply(2)
        torch.cuda.synchronize()
        a, b = trs["symm"].store, trs["nccl"].store
        res[f"{impl}_master"] = (a.master - b.master).abs().max().item()
        # compare bit patterns: fp32 tensors live as pairs of 16-bit units in the compute buffer
        res[f"{impl}_compute"] = float((a.compute.view(torch.int16) != b.compute.view(torch.int16)).sum().item())
        if impl == "cuda":
            ids = torch.randint(0, cfg.vocab_size, (2, 129), device=dev, generator=g)
            out = trs["symm"].train_step([{"input_ids": ids[:, :-1], "labels": ids[:, 1:]}])
            res["train_loss_finite"] = bool(torch.isfinite(out["loss"]).item())
        for tr in trs.values():
            tr.close()
    torch.save(res, os.path.join(outdir, f"rank{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_rank_fused_step_matches_nccl():
    import socket
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_worker, args=(2, port, d), nprocs=2, join=True)
        for r in range(2):
            res = torch.load(os.path.join(d, f"rank{r}.pt"))
            assert res["cuda_fused"] and not res["eager_fused"]
            # two ranks: a + b == b + a in fp32, so the two paths agree exactly
            for k in ("cuda_master", "cuda_compute", "eager_master", "eager_compute"):
                assert res[k] <= 1e-6, (r, k, res[k])
            assert res["train_loss_finite"]
