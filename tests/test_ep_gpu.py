"""Expert parallelism over NVLink peer memory (2 GPUs): the EP MoE equals the
single-GPU MoE holding all experts, for outputs, input / gate / shared gradients
and the expert weight gradients summed over the ranks' tokens.  Two routings: a
random one and one where every token picks rank 0's experts (rank 1 receives no
rows)."""
import os
import tempfile
from datetime import timedelta

import pytest
import torch

pytestmark = pytest.mark.gpu


def _worker(rank, world, port, outdir):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    from atomic_ai_hybrid_b200 import ops
    from atomic_ai_hybrid_b200.ops import kernels as K
    from atomic_ai_hybrid_b200.parallel.ep import EPGroup, moe_forward_ep
    ops.set_impl("cuda")
    T, d, F, E, k = 300, 256, 256, 8, 2
    El = E // world
    ep = EPGroup(world, rank, E, k, d, T, dev)
    res = {}
    for case in ("random", "rank0_only"):
        g = torch.Generator(device=dev).manual_seed(0)
        W = [(torch.randn(E, d, F, device=dev, generator=g) * d ** -0.5).to(torch.bfloat16),
             (torch.randn(E, F, d, device=dev, generator=g) * F ** -0.5).to(torch.bfloat16),
             (torch.randn(E, d, F, device=dev, generator=g) * d ** -0.5).to(torch.bfloat16)]
        gx = torch.Generator(device=dev).manual_seed(100 + rank)
        x = (torch.randn(T, d, device=dev, generator=gx) * 0.5).to(torch.bfloat16)
        logits = torch.randn(T, E, device=dev, generator=gx)
        if case == "rank0_only":
            logits[:, El:] = -1e4
        top = torch.topk(logits, k, -1).indices
        gate = torch.softmax(logits.gather(1, top), -1)
        shared = torch.randn(T, d, device=dev, generator=gx).to(torch.bfloat16)
        dy = torch.randn(T, d, device=dev, generator=gx).to(torch.bfloat16)
        runs = {}
        for mode in ("full", "ep"):
            xx, gg, ss = (t.clone().requires_grad_(True) for t in (x, gate, shared))
            if mode == "full":
                ws = [w.clone().requires_grad_(True) for w in W]
                out = K.moe_forward(xx, top, gg, ws[0], ws[1], ws[2], ss, "swiglu")
            else:
                ws = [w[rank * El:(rank + 1) * El].clone().requires_grad_(True) for w in W]
                out = moe_forward_ep(xx, top, gg, ws[0], ws[1], ws[2], ss, "swiglu", ep)
            out.backward(dy)
            runs[mode] = (out.float(), xx.grad.float(), gg.grad.float(), ss.grad.float(),
                          [w.grad.float() for w in ws])
        full, epr = runs["full"], runs["ep"]
        err = lambda a, b: float((a - b).abs().max() / (b.abs().max() + 1e-6))  # noqa: E731
        res[case] = {"out": err(epr[0], full[0]), "dx": err(epr[1], full[1]), "dgate": err(epr[2], full[2]),
                     "dshared": err(epr[3], full[3])}
        for i, (wf, wl) in enumerate(zip(full[4], epr[4])):
            dist.all_reduce(wf)  # every rank's tokens contribute to every expert
            res[case][f"dw{i + 1}"] = err(wl, wf[rank * El:(rank + 1) * El])
    ep.close()
    torch.save(res, os.path.join(outdir, f"rank{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_moe_matches_full_moe():
    import socket
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_worker, args=(2, port, d), nprocs=2, join=True)
        for r in range(2):
            res = torch.load(os.path.join(d, f"rank{r}.pt"))
            for case, errs in res.items():
                for key, v in errs.items():
                    assert v < 2e-2, (r, case, key, v)
