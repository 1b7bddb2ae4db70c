"""Benchmark configuration 1 end to end on the CPU in fp32 (its run file, its full size:
vocab 4096, d 256, 4 layers alternating Mamba2 / GDN-2, 8 experts top-2 of hidden 512,
batch 2 x 512): one forward / backward / AdamW step through the trainer, checked against
an independent restatement of the step -- the gradients of a plain autograd pass over the
same model, clipped to the global norm, then ``torch.optim.AdamW`` with the reference's
hyper-parameters (reference `optimizer.py:84-240`: b1 0.9, b2 0.999, eps 1e-8, decoupled
weight decay 0.01 on the decayed group, global clip 0.35)."""
import copy
import os

import torch

from atomic_ai_hybrid_b200.config import load_yaml_config
from atomic_ai_hybrid_b200.models import HybridMoEModel
from atomic_ai_hybrid_b200.optim.schedule import path_key
from atomic_ai_hybrid_b200.training.loss import compute_loss
from atomic_ai_hybrid_b200.training.trainer import Trainer

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
RUN_FILE = os.path.join(ROOT, "atomic_ai_hybrid_b200", "configs", "config1_tiny_cpu.yaml")


def test_config1_step_matches_plain_autograd_and_torch_adamw():
    cfg = load_yaml_config(RUN_FILE)
    assert (cfg.vocab_size, cfg.d_model, cfg.num_layers, cfg.e_routed, cfg.top_k, cfg.d_ff) == (4096, 256, 4, 8, 2, 512)
    torch.manual_seed(0)
    model = HybridMoEModel(cfg, compute_dtype=torch.float32)
    ref = copy.deepcopy(model)
    g = torch.Generator().manual_seed(1)
    ids = torch.randint(0, cfg.vocab_size, (2, 513), generator=g)
    batch = {"input_ids": ids[:, :-1], "labels": ids[:, 1:]}

    # the independent step: autograd gradients of the training loss (router terms
    # included; the run file has no router noise and no dropout), global clip, torch
    # AdamW per label group
    assert cfg.router_noise_std == 0.0 and getattr(cfg, "dropout_rate", 0.0) == 0.0
    ref.train()
    loss_ref, _ = compute_loss(ref, batch, deterministic=False)
    loss_ref.backward()
    tr = Trainer(model, total_steps=100, optimizer="adamw", compute_dtype=torch.float32, device=torch.device("cpu"))
    lrs = tr.opt.lrs(0)
    labels = {s.name: s.label for s in tr.store.segs}
    named = dict(ref.named_parameters())
    norm = torch.sqrt(sum((p.grad.double() ** 2).sum() for p in named.values() if p.grad is not None))
    coef = min(1.0, 0.35 / float(norm))
    checked = []
    for name, p in named.items():
        lab = labels[name]
        key = path_key(name)
        if not lab.startswith("adamw") or p.grad is None or "router_temp" in key or "expert_bias" in key:
            continue
        opt = torch.optim.AdamW([p], lr=lrs[lab], betas=(0.9, 0.999), eps=1e-8,
                                weight_decay=0.01 if lab == "adamw_decay" else 0.0)
        p.grad.mul_(coef)
        opt.step()
        checked.append(name)

    # the framework's step on the same batch
    out = tr.train_step([batch])
    assert torch.isfinite(out["loss"]) and bool(out["is_finite"])
    lr_ = float(loss_ref.detach())
    assert abs(float(out["loss"]) - lr_) <= 1e-5 * abs(lr_)
    assert abs(float(out["global_norm"]) - float(norm)) <= 1e-4 * float(norm)
    got = {n: p.detach() for n, p in model.named_parameters()}
    assert len(checked) > 20
    worst = max(float((got[n] - named[n].detach()).abs().max()) for n in checked)
    assert worst < 1e-5, worst
