"""Device-time breakdown of one training micro-step by kernel (PyTorch profiler / CUPTI).

    python -m atomic_ai_hybrid_b200.utils.stepprof --model hybrid_1b --micro-batch 4

Builds the benchmark model (random init), runs two warm-up optimizer steps, then profiles
one micro-step (forward, loss, backward, gradient accumulation) and prints every
kernel's total device time, launch count and share.  Times under a profiler are for
shares only; throughput figures come from ``bench.py``.
"""
from __future__ import annotations

import argparse

import torch


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="hybrid_1b")
    ap.add_argument("--micro-batch", type=int, default=4)
    ap.add_argument("--seq-len", type=int, default=4096)
    ap.add_argument("--top", type=int, default=60)
    ap.add_argument("--copies", action="store_true",
                    help="also list the PyTorch copy / contiguous / cat operators with their input shapes")
    a = ap.parse_args(argv)
    from .. import get_preset, ops
    from ..models import HybridMoEModel
    from ..training.trainer import Trainer
    ops.set_impl("cuda")
    dev = torch.device("cuda", 0)
    cfg = get_preset(a.model)
    with torch.device(dev):
        m = HybridMoEModel(cfg, compute_dtype=torch.bfloat16)
    with torch.no_grad():
        for n, p in m.named_parameters():
            if p.ndim >= 2 and "conv_w" not in n:
                p.normal_(0, 0.02)
    tr = Trainer(m, 1000, optimizer="adamw", device=dev)
    tr.opt.schedule.warmup = 1
    ids = torch.randint(0, cfg.vocab_size, (a.micro_batch, a.seq_len + 1), device=dev)
    b = [{"input_ids": ids[:, :-1], "labels": ids[:, 1:]}]
    for _ in range(2):
        tr.train_step(b)
    torch.cuda.synchronize()
    from torch.profiler import ProfilerActivity, profile
    acts = [ProfilerActivity.CUDA] + ([ProfilerActivity.CPU] if a.copies else [])
    with profile(activities=acts, record_shapes=a.copies) as prof:
        tr.micro_step(b[0])
        torch.cuda.synchronize()
    if a.copies:
        cops = [e for e in prof.key_averages(group_by_input_shape=True)
                if e.key in ("aten::copy_", "aten::contiguous", "aten::clone", "aten::cat", "aten::to",
                             "aten::_to_copy", "aten::reshape") and e.device_time_total > 0]
        for e in sorted(cops, key=lambda e: -e.device_time_total)[:30]:
            print(f"[copy] {e.device_time_total / 1000:8.2f} ms x{e.count:4d} {e.key} {e.input_shapes}")
    rows = sorted([(e.self_device_time_total, e.count, e.key) for e in prof.key_averages()
                   if e.self_device_time_total > 0], reverse=True)
    tot = sum(r[0] for r in rows)
    print(f"total device us {tot:.0f}")
    for t, c, k in rows[:a.top]:
        print(f"{t / 1000:9.2f} ms {100 * t / tot:5.1f}% x{c:5d}  {k[:110]}")
    tr.close()


if __name__ == "__main__":
    main()
