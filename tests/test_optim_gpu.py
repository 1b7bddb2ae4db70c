"""Fused optimizer kernels against the eager implementation of the same step."""
import pytest
import torch

from atomic_ai_hybrid_b200 import get_preset, ops
from atomic_ai_hybrid_b200.models import HybridMoEModel
from atomic_ai_hybrid_b200.optim import FlatParamStore, HybridOptimizer, grad_scale_of, label_of, label_adamw_only

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("labeler", [label_of, label_adamw_only])
def test_fused_step_matches_eager(labeler):
    cfg = get_preset("reference_tiny", d_model=256, n_heads=2, d_ff=256, num_experts=5)
    dev = torch.device("cuda", 0)
    stores, opts = [], []
    for impl in ("eager", "cuda"):
        torch.manual_seed(0)
        m = HybridMoEModel(cfg, compute_dtype=torch.bfloat16).to(dev)
        st = FlatParamStore(m, labeler, grad_scale_of, compute_dtype=torch.bfloat16, device=dev)
        opt = HybridOptimizer(st, total_steps=100)
        opt.schedule.warmup = 1
        stores.append(st)
        opts.append(opt)
    g = torch.Generator(device=dev).manual_seed(1)
    frac = torch.rand(cfg.num_blocks, cfg.e_routed, device=dev, generator=g) / cfg.e_routed * 2
    for step in range(3):
        grad = torch.randn(stores[0].grad.shape, device=dev, generator=g) * 0.01
        grad[5] = float("nan")
        for impl, st, opt in zip(("eager", "cuda"), stores, opts):
            st.grad.copy_(grad)
            with ops.impl(impl):
                info = opt.step(2, frac)
        for s0, s1 in zip(stores[0].segs, stores[1].segs):
            a, b = stores[0].master_view(s0), stores[1].master_view(s1)
            torch.testing.assert_close(b, a, rtol=2e-5, atol=2e-6, msg=s0.name)
            torch.testing.assert_close(stores[1].compute_view(s1).float(), stores[0].compute_view(s0).float(),
                                       rtol=1e-2, atol=1e-3)
    assert not bool(info["is_finite"])
