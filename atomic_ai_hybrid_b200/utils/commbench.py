"""NVLink collective paths against NCCL and against the link roofline (one node).

    torchrun --nproc-per-node N --master-addr 127.0.0.1 -m atomic_ai_hybrid_b200.utils.commbench

Each case is timed with CUDA events on the launching stream after warm-up, max over
ranks.  The roofline of a transfer is its bytes crossing NVLink per GPU (in or out,
whichever is larger) at the measured 770 GB/s per direction; a fused GEMM +
collective is bounded by the slower of that and its FLOPs at the measured bf16
GEMM throughput (``MEASURED_PEAKS.json``).  One JSON line per case on rank 0.

Cases:
  tp_all_gather   token rows, copy engines pulling from the peers' IPC buffers
  tp_reduce_scatter  partial rows pushed by the copy engines + slot sum
  tp_gemm_rs      tcgen05 GEMM whose epilogue stores partial tiles into the owners
  dp_reduce_scatter / dp_all_gather  the data-parallel fused-step transfers as
                  stand-alone kernels (fp32 gradient slice pull-sum, bf16 push)
  ep_dispatch / ep_return  expert-parallel token rows (uniform top-k routing) stored
                  into the expert owners' receive buffers and the results back
"""
from __future__ import annotations

import argparse
import json
import os
from datetime import timedelta

import torch
import torch.distributed as dist

LINK_GBS = 770.0


def _peaks():
    p = os.path.join(os.path.dirname(__file__), "..", "..", "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d.get("bf16_tflops", 1590.0))
    except Exception:
        return 1590.0


def _time(fn, warmup: int, iters: int) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / iters], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--rows", type=int, default=16384, help="token rows per rank")
    ap.add_argument("--width", type=int, default=4096)
    ap.add_argument("--k", type=int, default=512, help="contraction of the row-parallel GEMM (d_in / W)")
    ap.add_argument("--dp-mb", type=int, default=512, help="fp32 gradient MB per rank for the data-parallel cases")
    ap.add_argument("--ep-tokens", type=int, default=16384, help="tokens per rank for the expert-parallel cases")
    ap.add_argument("--ep-experts", type=int, default=64)
    ap.add_argument("--ep-k", type=int, default=4)
    ap.add_argument("--ep-d", type=int, default=2048)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--iters", type=int, default=10)
    args = ap.parse_args(argv)
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    W, rank = dist.get_world_size(), dist.get_rank()
    from ..ops._ext import ext
    from ..parallel.tp_peer import PeerTP
    E = ext()
    peak = _peaks()
    n, w = args.rows, args.width
    peer = PeerTP(W, rank, None, dev, n, w)
    out = []

    def emit(case, ms, nbytes, flops=0.0, nccl_ms=None, extra=None):
        t_link = nbytes / (LINK_GBS * 1e9) * 1e3
        t_gemm = flops / (peak * 1e12) * 1e3
        roof = max(t_link, t_gemm)
        rec = {"case": case, "world": W, "ms": round(ms, 4), "link_bytes_per_gpu": nbytes,
               "achieved_gbs": round(nbytes / (ms / 1e3) / 1e9, 1), "roofline_ms": round(roof, 4),
               "frac_of_roofline": round(roof / ms, 3)}
        if flops:
            rec["tflops"] = round(flops / (ms / 1e3) / 1e12, 1)
        if nccl_ms is not None:
            rec["nccl_ms"] = round(nccl_ms, 4)
        if extra:
            rec.update(extra)
        out.append(rec)
        if rank == 0:
            print(json.dumps(rec), flush=True)

    g = torch.Generator(device=dev).manual_seed(rank)
    x = torch.randn(n, w, device=dev, generator=g).to(torch.bfloat16)
    full = torch.empty(W * n, w, dtype=torch.bfloat16, device=dev)
    inbound = (W - 1) * n * w * 2
    ms = _time(lambda: peer.all_gather_rows(x), args.warmup, args.iters)
    nccl = _time(lambda: dist.all_gather_into_tensor(full, x), args.warmup, args.iters)
    emit("tp_all_gather", ms, inbound, nccl_ms=nccl)

    y = torch.randn(W * n, w, device=dev, generator=g).to(torch.bfloat16)
    part = torch.empty(n, w, dtype=torch.bfloat16, device=dev)
    ms = _time(lambda: peer.reduce_scatter_rows(y), args.warmup, args.iters)
    nccl = _time(lambda: dist.reduce_scatter_tensor(part, y), args.warmup, args.iters)
    emit("tp_reduce_scatter", ms, inbound, nccl_ms=nccl)

    a = torch.randn(W * n, args.k, device=dev, generator=g).to(torch.bfloat16)
    wt = (torch.randn(args.k, w, device=dev, generator=g) / args.k ** 0.5).to(torch.bfloat16)
    flops = 2.0 * W * n * args.k * w
    ms = _time(lambda: peer.gemm_rs(a, wt), args.warmup, args.iters)

    def unfused():
        p = a @ wt
        dist.reduce_scatter_tensor(part, p)

    nccl = _time(unfused, args.warmup, args.iters)
    gemm_only = _time(lambda: a @ wt, args.warmup, args.iters)
    emit("tp_gemm_rs", ms, inbound, flops, nccl_ms=nccl, extra={"cublas_gemm_ms": round(gemm_only, 4)})

    # data-parallel fused-step transfers as stand-alone kernels over IPC buffers
    nel = args.dp_mb * 1024 * 1024 // 4
    nel -= nel % (4 * W)
    ptr = E.ipc_alloc(nel * 4)
    cptr = E.ipc_alloc(nel * 2)
    try:
        mine = torch.cat([E.ipc_handle(ptr), E.ipc_handle(cptr)]).numpy().tobytes()
        allh = [None] * W
        dist.all_gather_object(allh, mine)
        gp, cp, opened = [], [], []
        for r in range(W):
            if r == rank:
                gp.append(ptr)
                cp.append(cptr)
                continue
            for i, lst in ((0, gp), (1, cp)):
                h = torch.frombuffer(bytearray(allh[r][64 * i:64 * (i + 1)]), dtype=torch.uint8)
                p = E.ipc_open(h)
                opened.append(p)
                lst.append(p)
        gpt = torch.tensor(gp, dtype=torch.int64, device=dev)
        cpt = torch.tensor(cp, dtype=torch.int64, device=dev)
        grad = E.ipc_tensor(ptr, nel, torch.empty(0, device=dev))
        grad.normal_()
        comp = E.ipc_tensor(cptr, nel, torch.empty(0, dtype=torch.bfloat16, device=dev))
        sl = nel // W
        lo = rank * sl
        dst = torch.empty(sl, device=dev)
        torch.cuda.synchronize()
        dist.barrier()
        ms = _time(lambda: E.reduce_scatter_f32(gpt, lo, dst), args.warmup, args.iters)
        g32 = torch.randn(nel, device=dev)
        o32 = torch.empty(sl, device=dev)
        nccl = _time(lambda: dist.reduce_scatter_tensor(o32, g32), args.warmup, args.iters)
        emit("dp_reduce_scatter", ms, (W - 1) * sl * 4, nccl_ms=nccl)
        src = comp[lo * 1:(lo + sl)]
        ms = _time(lambda: E.copy_out(src, cpt, lo * 2), args.warmup, args.iters)
        c16 = torch.empty(nel, dtype=torch.bfloat16, device=dev)
        nccl = _time(lambda: dist.all_gather_into_tensor(c16, src), args.warmup, args.iters)
        emit("dp_all_gather", ms, (W - 1) * sl * 2, nccl_ms=nccl)
        torch.cuda.synchronize()
        dist.barrier()
        for p in opened:
            E.ipc_close(p)
    finally:
        torch.cuda.synchronize()
        dist.barrier()
        E.ipc_free(ptr)
        E.ipc_free(cptr)
    peer.close()

    # expert parallelism: dispatch / return of routed rows (uniform routing, k distinct experts)
    from ..parallel.ep import EPGroup
    T, k, d, nE = args.ep_tokens, args.ep_k, args.ep_d, args.ep_experts
    ep = EPGroup(W, rank, nE, k, d, T, dev)
    scores = torch.rand(T, nE, device=dev, generator=g)
    top_idx = scores.topk(k, dim=1).indices.to(torch.int32).contiguous()
    xb = torch.randn(T, d, device=dev, generator=g).to(torch.bfloat16)
    eidx, counts, off_local, pos = E.moe_route_local(top_idx, nE)
    E.ep_publish(counts, ep.count_peers, ep.rank)
    ep.barrier()
    dst_base, off, seg, R = ep.layout()
    dst_pos = torch.empty(T * k, dtype=torch.int32, device=dev)
    cnt = counts.cpu().numpy().reshape(-1)
    El = nE // W
    remote_rows = int(cnt.sum() - cnt[rank * El:(rank + 1) * El].sum())

    def dispatch():
        E.ep_dispatch(xb, True, T, k, eidx, pos, off_local, dst_base, ep.El, ep.recv_peers, ep.meta_peers, ep.rank,
                      dst_pos)
        ep.barrier()

    ms = _time(dispatch, args.warmup, args.iters)
    emit("ep_dispatch", ms, remote_rows * (d * 2 + 8), extra={"rows_out": int(cnt.sum()), "remote_rows": remote_rows})
    meta = ep.meta[:R].clone()
    ys = torch.randn(R, d, device=dev, generator=g).to(torch.bfloat16)
    mine = meta[:, 0].cpu()
    back_remote = int((mine != rank).sum()) if R > 0 else 0

    def ret():
        if R > 0:
            E.ep_return(ys, meta, R, ep.ret_peers)
        ep.barrier()

    ms = _time(ret, args.warmup, args.iters)
    emit("ep_return", ms, max(back_remote, 1) * d * 2, extra={"rows_in": R, "remote_rows": back_remote})
    # the same exchange with NCCL: an all-to-all of the rows grouped by destination rank
    send = torch.randn(T * k, d, device=dev, generator=g).to(torch.bfloat16)
    per = [int(cnt[r * El:(r + 1) * El].sum()) for r in range(W)]
    recv_sizes = torch.tensor(per, dtype=torch.int64, device=dev)
    allsz = [torch.empty_like(recv_sizes) for _ in range(W)]
    dist.all_gather(allsz, recv_sizes)
    rin = [int(a[rank]) for a in allsz]
    rbuf = torch.empty(sum(rin), d, dtype=torch.bfloat16, device=dev)
    nccl = _time(lambda: dist.all_to_all_single(rbuf, send, rin, per), args.warmup, args.iters)
    out[-2]["nccl_all_to_all_ms"] = round(nccl, 4)
    if rank == 0:
        print(json.dumps({"case": "ep_nccl_all_to_all", "world": W, "ms": round(nccl, 4)}), flush=True)
    ep.close()
    dist.barrier()
    dist.destroy_process_group()
    return out


if __name__ == "__main__":
    main()
