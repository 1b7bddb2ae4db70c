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


def test_offloaded_moments_on_cuda(tmp_path):
    """``offload_moments`` with the store on the GPU: the moments live in pinned host memory,
    three steps give bit-identical parameters and moments to device moments on the same
    (eager) update path and match the fused kernel's step, and the host moments survive a
    checkpoint round trip."""
    from atomic_ai_hybrid_b200.ckpt.manager import CheckpointManager
    cfg = get_preset("reference_tiny", d_model=256, n_heads=2, d_ff=256, num_experts=5)
    dev = torch.device("cuda", 0)
    runs = {}
    for name, offload, impl in (("device_eager", False, "eager"), ("offload", True, "cuda"),
                                ("device_fused", False, "cuda")):
        torch.manual_seed(0)
        m = HybridMoEModel(cfg, compute_dtype=torch.bfloat16).to(dev)
        st = FlatParamStore(m, label_adamw_only, grad_scale_of, compute_dtype=torch.bfloat16, device=dev)
        opt = HybridOptimizer(st, total_steps=100, offload_moments=offload)
        opt.schedule.warmup = 1
        if offload:
            assert opt.m.device.type == "cpu" and opt.v.device.type == "cpu"
            assert opt.m.is_pinned() and opt.v.is_pinned()
            assert not opt.uses_kernels()
        g = torch.Generator(device=dev).manual_seed(1)
        for _ in range(3):
            st.grad.copy_(torch.randn(st.grad.shape, device=dev, generator=g) * 0.01)
            with ops.impl(impl):
                opt.step(1)
        torch.cuda.synchronize()
        runs[name] = (st, opt)
    (s0, o0), (s1, o1), (s2, o2) = runs["device_eager"], runs["offload"], runs["device_fused"]
    assert torch.equal(s1.master, s0.master)
    assert torch.equal(o1.m, o0.m.cpu()) and torch.equal(o1.v, o0.v.cpu())
    torch.testing.assert_close(s1.master, s2.master, rtol=2e-5, atol=2e-6)
    torch.testing.assert_close(o1.m, o2.m.cpu(), rtol=2e-5, atol=1e-9)

    class _T:  # the two attributes a checkpoint reads
        pass
    t = _T()
    t.store, t.opt = s1, o1
    CheckpointManager(str(tmp_path), "latest").save(3, t, asynchronous=False)
    m_ref, v_ref = o1.m.clone(), o1.v.clone()
    o1.m.zero_()
    o1.v.zero_()
    CheckpointManager(str(tmp_path), "latest").restore(3, t)
    assert torch.equal(o1.m, m_ref) and torch.equal(o1.v, v_ref)
    assert o1.m.device.type == "cpu" and o1.m.is_pinned() and o1.v.is_pinned()


def test_fused_step_with_bf16_gradients():
    """A store with bf16 gradient accumulators steps like one with fp32 accumulators holding
    the same (bf16-representable) gradients: the fused kernels read and scale either type."""
    cfg = get_preset("reference_tiny", d_model=256, n_heads=2, d_ff=256, num_experts=5)
    dev = torch.device("cuda", 0)
    runs, grads = [], None
    for gdt in (torch.float32, torch.bfloat16):
        torch.manual_seed(0)
        m = HybridMoEModel(cfg, compute_dtype=torch.bfloat16).to(dev)
        st = FlatParamStore(m, label_adamw_only, grad_scale_of, compute_dtype=torch.bfloat16, device=dev,
                            grad_dtype=gdt)
        assert st.grad.dtype == gdt
        if grads is None:
            g = torch.Generator(device=dev).manual_seed(4)
            grads = [(torch.randn(st.grad.numel(), device=dev, generator=g) * 0.01).to(torch.bfloat16)
                     for _ in range(3)]
        opt = HybridOptimizer(st, total_steps=100)
        opt.schedule.warmup = 1
        assert opt.uses_kernels()
        for gr in grads:
            st.grad.copy_(gr.to(gdt))
            with ops.impl("cuda"):
                opt.step(1)
        torch.cuda.synchronize()
        runs.append((st.master.clone(), opt.m.clone(), opt.v.clone()))
    for a, b in zip(*runs):
        torch.testing.assert_close(b, a, rtol=1e-2, atol=1e-6)


@pytest.mark.parametrize("shape", [(256, 512), (1024, 256), (4, 256, 768), (3, 1024, 512), (2, 2048, 1024),
                                   (96, 160)])
def test_muon_newton_schulz_on_tensor_cores(shape):
    """Muon's three Newton-Schulz steps on the grouped tcgen05 GEMM (bf16 operands, fp32 X)
    against the fp32 PyTorch iteration; (96, 160) takes the PyTorch path (sides off the tiles)."""
    from atomic_ai_hybrid_b200.ops import kernels as K, reference as R
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    lead, (a, b) = shape[:-2], shape[-2:]
    # a gradient-like matrix: a few strong directions over noise
    x = (torch.randn(*lead, a, 8, device=dev, generator=g) @ torch.randn(*lead, 8, b, device=dev, generator=g)
         + 0.1 * torch.randn(*shape, device=dev, generator=g))
    ref = R.newton_schulz3(x)
    out = K.newton_schulz3(x)
    assert out.shape == x.shape and out.dtype == torch.float32
    for i in range(out.reshape(-1, a, b).shape[0]):
        o, r = out.reshape(-1, a, b)[i], ref.reshape(-1, a, b)[i]
        assert ((o - r).norm() / r.norm()).item() < 2e-3, i
    # a non-finite gradient zeroes its matrix, as the reference's nan_to_num does
    x.view(-1, a, b)[0, 3, 5] = float("nan")
    out = K.newton_schulz3(x)
    assert torch.equal(out.reshape(-1, a, b)[0], torch.zeros(a, b, device=dev))
    assert torch.isfinite(out).all()
