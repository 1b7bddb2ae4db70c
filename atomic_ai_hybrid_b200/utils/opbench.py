"""Single-GPU operator benchmark (the scan-operator configuration): GDN-2 chunked
delta rule and Mamba2 SSD, forward + backward, bf16, timed with CUDA events; also
the MoE grouped FFN, the fused router, the fused residual/norm glue and conv1d.

``python -m atomic_ai_hybrid_b200.utils.opbench --op gdn --B 8 --T 4096 --H 16``
``python -m atomic_ai_hybrid_b200.utils.opbench --op ssd --B 8 --T 4096 --H 32``
``python -m atomic_ai_hybrid_b200.utils.opbench --op muon --B 32 --K 2048 --N 1024`` (Muon on 32 experts)

Inputs: GDN q, k ~ N(0,1) then L2-normalised per head, v ~ N(0,1),
beta = sigmoid(N(0,1)), g = -softplus(N(0,1)) (per head, broadcast over the
channels of the per-channel kernels; erase gate = beta, write gate = 1).  SSD x, B,
C ~ N(0,1), dt = softplus(N(0,1) - 4) per head (broadcast over channels),
A = -exp(U[0, log 16]).  Reported TFLOP/s count the chunked algorithm's matmul
FLOPs (``ops.reference.flops_*``; backward counted as 2x forward).  Between timed
iterations a 256 MiB buffer is rewritten to flush L2.
"""
from __future__ import annotations

import argparse
import json
import math

import torch
import torch.nn.functional as F


def _timeit(fn, warmup: int, iters: int, flush: torch.Tensor) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b))
    times.sort()
    return times[len(times) // 2]


# per-phase cycle counters of the scan kernels (csrc/phase_prof.cuh): slot base, phase names; names
# starting with "@" are per-warp arrival times, not phases of the sum
_PHASES = {
    "ssd_chunk_fwd_tc": (0, ["setup", "load wait", "cumsum + V", "CB out", "y_diag blocks", "MMA wait", "YD rows",
                             "diagonal blocks", "rows out"]),
    "ssd_chunk_bwd_tc": (16, ["setup + CB", "head loads", "cumsum", "phase-1 tiles", "-", "dCB MMA wait",
                              "dCB readout", "ddd blocks", "diagonal ddd", "MMA wait", "pass 1", "pass 2",
                              "row stores", "dC / dB", "dCB operands + MMA issue"]),
    # summed over the chunk steps
    "ssd_state_fwd_tc": (32, ["S out + previous y rows", "yd loads + state carry", "y_off MMA wait",
                              "y epilogue"]),
    "gdn_chunk_fwd_tc": (64, ["setup + g", "cumsum", "rows + score MMAs", "score wait", "scores out",
                              "inverse + w v tile", "sync + A image", "w~ / u MMA", "w~ / u out", "bk tile",
                              "@warp 0 at inverse sync", "@warp 1 at inverse sync", "@warp 2 at inverse sync",
                              "@warp 3 at inverse sync"]),
    "gdn_chunk_bwd_tc": (80, ["loads", "state products", "WV / dw~ / Gqk out", "WY wait", "dA out", "dv / dw",
                              "T, A^T T", "Gkk out", "intra blocks", "intra wait", "plain tiles", "assembly"]),
    # summed over the chunk steps; "load wait" (thread 0 waiting for the tiles) precedes the first MMA
    "gdn_state_fwd_tc": (96, ["h out", "V, O1 MMA", "v_new out", "O2, HH MMA", "o out", "h update",
                              "load wait"]),
    "gdn_state_bwd_tc": (112, ["dh out", "DVN, D1 MMA", "dv_new out", "D2 MMA", "-", "dh update", "load wait"]),
}


def _phase_report(fn, prefix):
    """One call of ``fn`` with the scan kernels' phase counters on: mean SM cycles per CTA of
    every phase of the kernels whose name starts with ``prefix``."""
    from ..ops._ext import ext
    cnt = torch.zeros(128, dtype=torch.int64, device="cuda")
    torch.cuda.synchronize()
    ext().phase_prof(cnt)
    try:
        fn()
        torch.cuda.synchronize()
    finally:
        ext().phase_prof(None)
    c = cnt.cpu().tolist()
    out = {}
    for name, (base, phases) in _PHASES.items():
        if not name.startswith(prefix):
            continue
        ctas = c[base + 15]
        if not ctas:
            continue
        cyc = [c[base + i] / ctas for i in range(len(phases))]
        tot = sum(v for p, v in zip(phases, cyc) if not p.startswith("@"))
        out[name] = {"ctas": ctas, "cycles_per_cta": round(tot),
                     "phases": {p: [round(v), round(v / tot, 3)] for p, v in zip(phases, cyc)}}
    return out


def bench_gdn(B, T, H, warmup, iters, flush, mode="fwdbwd", phases=False, impl="cuda"):
    from ..ops import kernels as K, reference as R
    from ..ops.reference import flops_gdn_chunked
    D = 128
    dev = "cuda"
    q = F.normalize(torch.randn(B, T, H, D, device=dev), dim=-1).to(torch.bfloat16).requires_grad_(True)
    k = F.normalize(torch.randn(B, T, H, D, device=dev), dim=-1).to(torch.bfloat16).requires_grad_(True)
    v = torch.randn(B, T, H, D, device=dev).to(torch.bfloat16).requires_grad_(True)
    beta = torch.sigmoid(torch.randn(B, T, H, 1, device=dev)).expand(B, T, H, D).contiguous()
    b = beta.to(torch.bfloat16).requires_grad_(True)
    w = torch.ones(B, T, H, D, device=dev, dtype=torch.bfloat16).requires_grad_(True)
    g = (-F.softplus(torch.randn(B, T, H, 1, device=dev))).expand(B, T, H, D).contiguous().requires_grad_(True)
    do = torch.randn(B, T, H, D, device=dev, dtype=torch.bfloat16)

    def run():
        if impl == "eager":  # the PyTorch chunked scan (checkpointed chunks), the eager baseline
            o = R.gdn2_chunked(q, k, v, g, b, w, 1.0, 64, checkpoint_chunks=True)[0]
        else:
            o = K.gdn2(q, k, v, w, b, g, 1.0, 64)
        if mode == "fwdbwd":
            torch.autograd.backward(o, do)

    ms = _timeit(run, warmup, iters, flush)
    fl = flops_gdn_chunked(B, T, H, D, 64) * (3 if mode == "fwdbwd" else 1)
    io_bytes = B * T * H * D * (2 * 5 + 4) * (3 if mode == "fwdbwd" else 1)
    r = {"op": "gdn2", "impl": impl, "mode": mode, "B": B, "T": T, "H": H, "D": D, "ms": ms, "tflops": fl / ms / 1e9,
         "min_io_gb_s": io_bytes / ms / 1e6}
    if phases:
        r["phases"] = _phase_report(run, "gdn")
    return r


def bench_ssd(B, T, H, warmup, iters, flush, mode="fwdbwd", phases=False, impl="cuda"):
    from ..ops import kernels as K, reference as R
    from ..ops.reference import flops_ssd_chunked
    P, N = 64, 128
    dev = "cuda"
    x = torch.randn(B, T, H, P, device=dev).to(torch.bfloat16).requires_grad_(True)
    dt = F.softplus(torch.randn(B, T, H, 1, device=dev) - 4).clamp(1e-2, 1.0).expand(B, T, H, P).contiguous()
    dt = dt.to(torch.bfloat16).requires_grad_(True)
    A = (-torch.exp(torch.rand(H, device=dev) * math.log(16.0))).requires_grad_(True)
    Bm = torch.randn(B, T, N, device=dev).to(torch.bfloat16).requires_grad_(True)
    Cm = torch.randn(B, T, N, device=dev).to(torch.bfloat16).requires_grad_(True)
    dy = torch.randn(B, T, H, P, device=dev, dtype=torch.bfloat16)

    def run():
        if impl == "eager":
            y = R.ssd_chunked(dt, A, Bm, Cm, x, 64, checkpoint_chunks=True)[0]
        else:
            y = K.ssd(dt, A, Bm, Cm, x, 64)
        if mode == "fwdbwd":
            torch.autograd.backward(y, dy)

    ms = _timeit(run, warmup, iters, flush)
    fl = flops_ssd_chunked(B, T, H, P, N, 64) * (3 if mode == "fwdbwd" else 1)
    io_bytes = (B * T * H * P * 2 * 3 + B * T * N * 2 * 2) * (3 if mode == "fwdbwd" else 1)
    r = {"op": "ssd", "impl": impl, "mode": mode, "B": B, "T": T, "H": H, "P": P, "N": N, "ms": ms, "tflops": fl / ms / 1e9,
         "min_io_gb_s": io_bytes / ms / 1e6}
    if phases:
        r["phases"] = _phase_report(run, "ssd")
    return r


def bench_moe(T, d, F_, E, k, warmup, iters, flush, mode="fwdbwd"):
    from ..ops import kernels as K
    dev = "cuda"
    x = (torch.randn(T, d, device=dev) * 0.5).to(torch.bfloat16).requires_grad_(True)
    logits = torch.randn(T, E, device=dev)
    top_idx = torch.topk(logits, k, -1).indices
    gate = torch.softmax(logits.gather(1, top_idx), -1).requires_grad_(True)
    w1 = (torch.randn(E, d, F_, device=dev) * d ** -0.5).to(torch.bfloat16).requires_grad_(True)
    w2 = (torch.randn(E, F_, d, device=dev) * F_ ** -0.5).to(torch.bfloat16).requires_grad_(True)
    w3 = (torch.randn(E, d, F_, device=dev) * d ** -0.5).to(torch.bfloat16).requires_grad_(True)
    dy = torch.randn(T, d, device=dev, dtype=torch.bfloat16)

    def run():
        y = K.moe_forward(x, top_idx, gate, w1, w2, w3, None, "swiglu")
        if mode == "fwdbwd":
            torch.autograd.backward(y, dy)

    ms = _timeit(run, warmup, iters, flush)
    fl = 2 * T * k * d * F_ * 3 * (3 if mode == "fwdbwd" else 1)
    return {"op": "moe_swiglu", "mode": mode, "T": T, "d": d, "F": F_, "E": E, "k": k, "ms": ms,
            "tflops": fl / ms / 1e9}


def bench_router(T, d, E, k, warmup, iters, flush, mode="fwdbwd"):
    """Fused MoE router (fp32-exact logits on tensor cores) forward (+ backward)."""
    from ..ops import kernels as K
    dev = "cuda"
    x = (torch.randn(T, d, device=dev) * 2).to(torch.bfloat16).requires_grad_(True)
    kern = torch.randn(d, E, device=dev)
    kn = (kern / kern.norm(dim=0, keepdim=True)).requires_grad_(True)
    temp = torch.full((1,), 10.0, device=dev, requires_grad=True)
    bias = torch.zeros(E, device=dev)

    def run():
        gate, psum, lse_sq, _, _, _ = K.router(x, kn, temp, bias, None, k)
        if mode == "fwdbwd":
            (gate.sum() + psum.square().sum() + lse_sq.sum()).backward()

    ms = _timeit(run, warmup, iters, flush)
    fl = 2 * T * d * E * 3 * (3 if mode == "fwdbwd" else 1)
    return {"op": "router", "mode": mode, "T": T, "d": d, "E": E, "k": k, "ms": ms,
            "min_io_gb_s": T * d * 2 * (3 if mode == "fwdbwd" else 1) / ms / 1e6, "tflops": fl / ms / 1e9}


def bench_attn(B, T, H, D, warmup, iters, flush, mode="fwdbwd"):
    """Causal flash attention (``attention.cu``) on (B, H, T, D) bf16."""
    from ..ops import kernels as K
    dev = "cuda"
    q, k, v = (torch.randn(B, H, T, D, device=dev).to(torch.bfloat16).requires_grad_(True) for _ in range(3))
    do = torch.randn(B, H, T, D, device=dev, dtype=torch.bfloat16)

    def run():
        o = K.attention(q, k, v, D ** -0.5)
        if mode == "fwdbwd":
            torch.autograd.backward(o, do)

    ms = _timeit(run, warmup, iters, flush)
    fl = 2 * B * H * T * T * D * (1 if mode == "fwd" else 3.5)  # causal: QK^T and PV at half; backward 2.5x
    return {"op": "attention", "mode": mode, "B": B, "T": T, "H": H, "D": D, "ms": ms, "tflops": fl / ms / 1e9}


def bench_ce(T, d, V, warmup, iters, flush, mode="fwdbwd"):
    """Tied LM head + label-smoothed cross entropy (no stored logits)."""
    from ..ops import kernels as K
    dev = "cuda"
    h = (torch.randn(T, d, device=dev) * 0.5).to(torch.bfloat16).requires_grad_(True)
    W = (torch.randn(V, d, device=dev) * 0.02).to(torch.bfloat16).requires_grad_(True)
    labels = torch.randint(0, V, (T,), device=dev)

    def run():
        s, c = K.cross_entropy(h, labels, W, 0.1)
        if mode == "fwdbwd":
            (s / c).backward()

    ms = _timeit(run, warmup, iters, flush)
    fl = 2 * T * d * V * (1 if mode == "fwd" else 4)  # forward logits; backward recomputes them, dh, dW
    return {"op": "ce", "mode": mode, "T": T, "d": d, "V": V, "ms": ms, "tflops": fl / ms / 1e9}


def bench_glue(T, d, warmup, iters, flush, mode="fwdbwd"):
    """Residual add + clip + RMSNorm and RMSNorm x SiLU gate (fused row kernels)."""
    from ..ops import kernels as K
    dev = "cuda"
    x = torch.randn(T, d, device=dev).to(torch.bfloat16).requires_grad_(True)
    delta = torch.randn(T, d, device=dev).to(torch.bfloat16).requires_grad_(True)
    z = torch.randn(T, d, device=dev).to(torch.bfloat16).requires_grad_(True)
    scale = torch.ones(d, device=dev, requires_grad=True)

    def run():
        xo, y = K.add_rmsnorm(x, delta, scale, 1e3, 1e-6, sanitize_delta_grad=True)
        o = K.norm_gate(y, z, scale, 1e-6, 1e2)
        if mode == "fwdbwd":
            torch.autograd.backward([o, xo], [torch.ones_like(o), torch.ones_like(xo)])

    ms = _timeit(run, warmup, iters, flush)
    # forward 6 row passes (x, delta, xo, y | y, z, o), backward 11
    io = T * d * 2 * (6 + (11 if mode == "fwdbwd" else 0))
    return {"op": "glue", "mode": mode, "T": T, "d": d, "ms": ms, "min_io_gb_s": io / ms / 1e6}


def bench_conv(B, T, C, warmup, iters, flush, mode="fwdbwd"):
    """Depthwise causal conv1d (width 4) + SiLU, streaming bf16 kernels."""
    from ..ops import kernels as K
    dev = "cuda"
    x = torch.randn(B, T, C, device=dev).to(torch.bfloat16).requires_grad_(True)
    w = (torch.randn(C, 4, device=dev) * 0.3).requires_grad_(True)
    b = torch.zeros(C, device=dev, requires_grad=True)
    dy = torch.randn(B, T, C, device=dev).to(torch.bfloat16)

    def run():
        y = K.conv1d(x, w, b, True, None)
        if mode == "fwdbwd":
            y.backward(dy)

    ms = _timeit(run, warmup, iters, flush)
    io = B * T * C * 2 * (2 + (3 if mode == "fwdbwd" else 0))
    return {"op": "conv1d", "mode": mode, "B": B, "T": T, "C": C, "ms": ms, "min_io_gb_s": io / ms / 1e6}


def bench_gemm(M, K, N, warmup, iters, flush):
    """C = A B^T at one shape: the single-CTA and CTA-pair tcgen05 kernels and cuBLAS."""
    from ..ops._ext import ext
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(N, K, device="cuda", dtype=torch.bfloat16)
    fl = 2.0 * M * K * N
    out = {"op": "gemm", "M": M, "K": K, "N": N}
    for name, fn in (("single_cta", lambda: ext().gemm_dense(a, b, pair=False)),
                     ("cta_pair", lambda: ext().gemm_dense(a, b, pair=True)),
                     ("cublas", lambda: torch.mm(a, b.t()))):
        ms = _timeit(fn, warmup, iters, flush)
        out[name] = {"ms": ms, "tflops": fl / ms / 1e9}
    # weight gradient of a projection K -> N over M tokens, added into an fp32 accumulator
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    dy = torch.randn(M, N, device="cuda", dtype=torch.bfloat16)
    acc = torch.zeros(K, N, device="cuda", dtype=torch.float32)
    for name, fn in (("wgrad_tcgen05", lambda: ext().dense_wgrad(x, dy, acc)),
                     ("wgrad_cublas", lambda: torch.addmm(acc, x.t(), dy, out_dtype=torch.float32, out=acc))):
        ms = _timeit(fn, warmup, iters, flush)
        out[name] = {"ms": ms, "tflops": fl / ms / 1e9}
    return out


def bench_gemm_rs(W, n, K, N, warmup, iters, flush):
    """The tensor-parallel GEMM + reduce-scatter kernel on one GPU: the W destination
    slots are local buffers (the NVLink stores become local stores), so this measures
    the GEMM and its staged epilogue; ``utils.commbench`` measures it across GPUs."""
    from ..ops._ext import ext
    E = ext()
    dev = "cuda"
    a = torch.randn(W * n, K, device=dev).to(torch.bfloat16)
    w = (torch.randn(K, N, device=dev) / K ** 0.5).to(torch.bfloat16)
    outs = [torch.empty(n, N, dtype=torch.bfloat16, device=dev) for _ in range(W)]
    off = torch.arange(W + 1, dtype=torch.int32, device=dev) * n
    ptrs = [o.data_ptr() for o in outs]
    ms = _timeit(lambda: E.tp_gemm_rs(a, w, off, ptrs, 0), warmup, iters, flush)
    fl = 2.0 * W * n * K * N
    return {"op": "gemm_rs_local", "W": W, "rows": W * n, "K": K, "N": N, "ms": ms, "tflops": fl / ms / 1e9}


def bench_muon(E, a, b, warmup, iters, flush):
    """Muon's three Newton-Schulz steps on E matrices of a x b (fp32 gradients): the grouped
    tcgen05 path against the fp32 PyTorch iteration.  FLOPs: 3 steps x two products of
    2 r^2 c each (r, c the shorter and longer side) per matrix."""
    from ..ops import kernels as K, reference as R
    g = torch.randn(E, a, b, device="cuda", dtype=torch.float32)
    r, c = min(a, b), max(a, b)
    fl = 3 * 2 * 2.0 * r * r * c * E
    out = {"op": "muon_ns", "E": E, "a": a, "b": b}
    for name, fn in (("tcgen05", lambda: K.newton_schulz3(g)), ("torch_fp32", lambda: R.newton_schulz3(g))):
        ms = _timeit(fn, warmup, iters, flush)
        out[name] = {"ms": ms, "tflops": fl / ms / 1e9}
    return out


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--op", default="gdn",
                    choices=["gdn", "ssd", "moe", "router", "glue", "conv", "gemm_rs", "gemm", "attn", "ce", "muon"])
    ap.add_argument("--K", type=int, default=2048)
    ap.add_argument("--N", type=int, default=2048)
    ap.add_argument("--mode", default="fwdbwd", choices=["fwd", "fwdbwd"])
    ap.add_argument("--B", type=int, default=8)
    ap.add_argument("--T", type=int, default=4096)
    ap.add_argument("--H", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--impl", default="cuda", choices=["cuda", "eager"],
                    help="gdn / ssd: the sm_100a kernels or the PyTorch chunked scans (eager baseline)")
    ap.add_argument("--phases", action="store_true",
                    help="gdn / ssd: also report the scan kernels' per-phase cycles (one extra call)")
    a = ap.parse_args(argv)
    from .. import ops
    ops.set_impl("cuda")
    flush = torch.empty(256 * 1024 * 1024 // 4, device="cuda", dtype=torch.float32)
    torch.manual_seed(0)
    if a.op == "gdn":
        r = bench_gdn(a.B, a.T, a.H or 16, a.warmup, a.iters, flush, a.mode, a.phases, a.impl)
    elif a.op == "ssd":
        r = bench_ssd(a.B, a.T, a.H or 32, a.warmup, a.iters, flush, a.mode, a.phases, a.impl)
    elif a.op == "moe":
        r = bench_moe(a.B * a.T, 2048, 1024, 32, 4, a.warmup, a.iters, flush, a.mode)
    elif a.op == "router":
        r = bench_router(a.B * a.T, 2048, 32, 4, a.warmup, a.iters, flush, a.mode)
    elif a.op == "glue":
        r = bench_glue(a.B * a.T, 2048, a.warmup, a.iters, flush, a.mode)
    elif a.op == "attn":
        r = bench_attn(a.B, a.T, a.H or 16, 128, a.warmup, a.iters, flush, a.mode)
    elif a.op == "ce":
        r = bench_ce(a.B * a.T, a.K, 50304, a.warmup, a.iters, flush, a.mode)
    elif a.op == "gemm":
        r = bench_gemm(a.B * a.T, a.K, a.N, a.warmup, a.iters, flush)
    elif a.op == "muon":
        r = bench_muon(a.B, a.K, a.N, a.warmup, a.iters, flush)
    elif a.op == "gemm_rs":
        r = bench_gemm_rs(2, a.B * a.T // 2, 512, 4096, a.warmup, a.iters, flush)
    else:
        r = bench_conv(a.B, a.T, 2048, a.warmup, a.iters, flush, a.mode)
    print(json.dumps(r), flush=True)
    return r


if __name__ == "__main__":
    main()
