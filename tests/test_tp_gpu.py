"""Tensor parallelism over NVLink peer memory.

One GPU: the GEMM with the reduce-scatter epilogue (every "rank" a local buffer in
the output table) and the slot sum, against PyTorch fp32 references.
Two GPUs: the peer all-gather / reduce-scatter / GEMM-reduce-scatter against NCCL,
and a head-split model (sm_100a kernels) against the single-rank model.
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


@pytest.mark.parametrize("W,n,K,N", [(2, 256, 512, 1024), (4, 128, 256, 544), (8, 128, 128, 256)])
def test_gemm_rs_epilogue_routes_rows_to_owners(W, n, K, N):
    E = _ext()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(W)
    a = torch.randn(W * n, K, device=dev, generator=g).to(torch.bfloat16)
    w = (torch.randn(K, N, device=dev, generator=g) / K ** 0.5).to(torch.bfloat16)
    outs = [torch.full((n, N), float("nan"), dtype=torch.bfloat16, device=dev) for _ in range(W)]
    off = torch.arange(W + 1, dtype=torch.int32, device=dev) * n
    for m_rot in (0, n // 128):
        E.tp_gemm_rs(a, w, off, [o.data_ptr() for o in outs], m_rot)
        torch.cuda.synchronize()
        assert E.gemm_error() == 0
        ref = a.float() @ w.float()
        for r in range(W):
            torch.testing.assert_close(outs[r].float(), ref[r * n:(r + 1) * n], rtol=2e-2, atol=2e-2)


def test_sum_slots():
    E = _ext()
    dev = torch.device("cuda", 0)
    W, n, stride = 3, 4096, 8192
    buf = torch.randn(W * stride, device=dev).to(torch.bfloat16)
    out = torch.empty(n, dtype=torch.bfloat16, device=dev)
    E.sum_slots(buf.data_ptr(), W, stride, out)
    ref = sum(buf[s * stride:s * stride + n].float() for s in range(W))
    torch.testing.assert_close(out.float(), ref, rtol=1e-2, atol=1e-2)


# ---------------------------------------------------------------- two ranks

def _cfg():
    from atomic_ai_hybrid_b200 import get_preset
    return get_preset("hybrid_1b", d_model=512, n_heads=4, n_heads_ssm=8, num_layers=2, d_ff=256,
                      n_routed_experts=8, top_k=2, vocab_size=1024, d_state=128, router_noise_std=0.0,
                      layer_types=("gdn2", "mamba2"))


def _cos(a, b):
    a, b = a.float().reshape(-1), b.float().reshape(-1)
    return float((a @ b) / (a.norm() * b.norm()).clamp_min(1e-30))


def _worker(rank, world, port, outdir):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    from atomic_ai_hybrid_b200 import ops
    from atomic_ai_hybrid_b200.models import HybridMoEModel
    from atomic_ai_hybrid_b200.parallel.context import ParallelContext, set_parallel_context
    from atomic_ai_hybrid_b200.parallel.tp import init_tensor_parallel, load_full_state, shard_spec, shard_tensor
    from atomic_ai_hybrid_b200.training.loss import compute_loss
    ops.set_impl("cuda")
    res = {}
    cfg = _cfg()
    B, L = 2, 256
    # ---- single-rank model (every rank computes it)
    set_parallel_context(ParallelContext())
    torch.manual_seed(0)
    full = HybridMoEModel(cfg, compute_dtype=torch.bfloat16).to(dev)
    ids = torch.randint(0, cfg.vocab_size, (B, L + 1), device=dev, generator=torch.Generator(device=dev).manual_seed(5))

    def run(m):
        m.zero_grad(set_to_none=True)
        loss, _ = compute_loss(m, {"input_ids": ids[:, :-1], "labels": ids[:, 1:]})
        loss.backward()
        return loss.detach(), {n: p.grad for n, p in m.named_parameters() if p.grad is not None}

    lf, gf = run(full)
    # ---- peer primitives against NCCL
    tp = init_tensor_parallel(world, dev, max_rows=B * L // world, max_width=cfg.d_model)
    peer = tp.peer
    res["has_peer"] = peer is not None
    n, w = B * L // world, cfg.d_model
    g = torch.Generator(device=dev).manual_seed(11 + rank)
    x = torch.randn(n, w, device=dev, generator=g).to(torch.bfloat16)
    ref = torch.empty(world * n, w, dtype=torch.bfloat16, device=dev)
    dist.all_gather_into_tensor(ref, x)
    res["ag"] = float((peer.all_gather_rows(x) - ref).abs().max())
    y = torch.randn(world * n, w, device=dev, generator=g).to(torch.bfloat16)
    ref = torch.empty(n, w, device=dev)
    dist.reduce_scatter_tensor(ref, y.float())
    res["rs"] = float((peer.reduce_scatter_rows(y).float() - ref).abs().max() / ref.abs().max())
    a = torch.randn(world * n, 256, device=dev, generator=g).to(torch.bfloat16)
    wt = (torch.randn(256, w, device=dev, generator=g) / 16).to(torch.bfloat16)
    dist.reduce_scatter_tensor(ref, a.float() @ wt.float())
    res["gemm_rs"] = float((peer.gemm_rs(a, wt).float() - ref).abs().max() / ref.abs().max())
    # ---- head-split model
    tpm = HybridMoEModel(cfg, compute_dtype=torch.bfloat16).to(dev)
    load_full_state(tpm, {k: v.float() for k, v in full.state_dict().items()})
    lt, gt = run(tpm)
    lsum = lt.clone()
    dist.all_reduce(lsum)
    res["loss"] = float((lsum / world - lf).abs() / lf.abs())
    # router matrices have the noisiest gradients (top-k near-ties and atomic accumulation
    # move tokens between experts): they are held to a looser bound, as in the parity test
    worst, worst_router, worst_name = 1.0, 1.0, None
    for name, p in tpm.named_parameters():
        if name not in gt or name not in gf:
            continue
        spec = shard_spec(p)
        if spec is not None:
            refg = shard_tensor(gf[name].float(), spec[0], spec[1], world, rank)
            got = gt[name].float()
        else:
            got = gt[name].float().clone()
            dist.all_reduce(got)
            refg = gf[name].float()
        if refg.norm() < 1e-6:
            continue
        if name.endswith("router_temp"):
            continue  # one scalar summing cancelling terms; its kernel is checked in test_kernels_fused
        c = _cos(got, refg)
        if name.endswith(".router") or refg.numel() <= 64:  # router matrices, per-head scalars
            worst_router = min(worst_router, c)
        elif c < worst:
            worst, worst_name = c, name
    res["grad_cos"], res["grad_cos_name"], res["router_cos"] = worst, worst_name, worst_router
    tp.close()
    set_parallel_context(ParallelContext())
    torch.save(res, os.path.join(outdir, f"rank{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_rank_tensor_parallel():
    import socket
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_worker, args=(2, port, d), nprocs=2, join=True)
        for r in range(2):
            res = torch.load(os.path.join(d, f"rank{r}.pt"))
            assert res["has_peer"]
            assert res["ag"] == 0.0, res
            assert res["rs"] < 1e-2 and res["gemm_rs"] < 2e-2, res
            assert res["loss"] < 2e-2, res
            assert res["grad_cos"] > 0.98, res
            assert res["router_cos"] > 0.9, res
