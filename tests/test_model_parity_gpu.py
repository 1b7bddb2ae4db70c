"""Whole-model parity: the sm_100a path (fused layers, tcgen05 MoE, fused router, CE)
against the eager PyTorch path on the same bf16 weights and batch -- loss,
activations after every sublayer and MoE, and every parameter gradient."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _run(impl, m, batch):
    from atomic_ai_hybrid_b200 import ops
    from atomic_ai_hybrid_b200.training.loss import compute_loss
    ops.set_impl(impl)
    m.zero_grad(set_to_none=True)
    acts, hooks = {}, []
    for name, mod in m.named_modules():
        if name.endswith(".sublayer") or name.endswith(".moe") or name.endswith(".intra"):
            def hk(mod, inp, out, name=name):
                acts[name] = out.detach().float().clone()
            hooks.append(mod.register_forward_hook(hk))
    loss, _ = compute_loss(m, batch, deterministic=False)
    loss.backward()
    for h in hooks:
        h.remove()
    grads = {n: p.grad.detach().float().clone() for n, p in m.named_parameters() if p.grad is not None}
    ops.set_impl("cuda")
    return float(loss), acts, grads


@pytest.mark.parametrize("arch,ffn_act,shared", [("interleaved", "swiglu", 1), ("interleaved", "gelu", 1),
                                                 ("interleaved", "swiglu", 0), ("blockdar", "swiglu", 1)])
def test_kernel_path_matches_eager_path(arch, ffn_act, shared):
    from atomic_ai_hybrid_b200 import get_preset
    from atomic_ai_hybrid_b200.models import HybridMoEModel
    dev = torch.device("cuda", 0)
    extra = {}
    if arch == "blockdar":  # every sublayer kind, BlockDAR source mixing, MLA on the attention kernel
        extra = dict(arch="blockdar", num_layers=3, layers_per_block=3, layer_types=("gdn2", "mamba2", "mla"),
                     d_latent=256)
    kw = dict(d_model=512, n_heads=4, n_heads_ssm=8, num_layers=2, d_ff=256, n_routed_experts=8, top_k=2,
              vocab_size=1024, d_state=128, router_noise_std=0.0, layer_types=("gdn2", "mamba2"),
              ffn_act=ffn_act, n_shared_experts=shared)
    kw.update(extra)
    cfg = get_preset("hybrid_1b", **kw)
    torch.manual_seed(0)
    m = HybridMoEModel(cfg, compute_dtype=torch.bfloat16).to(dev)
    for p in m.parameters():
        if p.ndim >= 2:
            p.data = p.data.to(torch.bfloat16)
    ids = torch.randint(0, cfg.vocab_size, (4, 257), device=dev, generator=torch.Generator(device=dev).manual_seed(1))
    batch = {"input_ids": ids[:, :-1], "labels": ids[:, 1:]}
    lk, ak, gk = _run("cuda", m, batch)
    le, ae, ge = _run("eager", m, batch)
    assert abs(lk - le) < 1e-2 * abs(le), (lk, le)
    # the two paths round differently (bf16 kernels vs partly-fp32 eager scans) and a few
    # near-tie tokens pick other experts, so later layers drift apart by several percent; a
    # wrong operation shows up as tens of percent (the shared-expert bug this test was
    # written for gave 54-97 %)
    for n, b in ae.items():
        rel = float((ak[n] - b).norm() / (b.norm() + 1e-12))
        first = n.startswith("layer_0.") or n.startswith("block_0.layer_0.")
        assert rel < (0.1 if first else 0.35), (n, rel)
    assert gk.keys() == ge.keys()
    for n, b in ge.items():
        a = gk[n].reshape(-1)
        b = b.reshape(-1)
        if b.norm() < 1e-8:
            continue
        cos = float(a @ b / (a.norm() * b.norm()))
        ratio = float(a.norm() / b.norm())
        if n.endswith("router_temp"):
            continue  # one scalar summing cancelling terms; its kernel is checked in test_kernels_fused
        if b.numel() <= 64:  # per-head scalars: sums over every token and channel
            assert cos > 0.9 and abs(ratio - 1) < 0.6, (n, cos, ratio)
        elif n.endswith(".router"):
            # the router kernel's gradient changes discontinuously where a near-tie token picks
            # another expert, and the kernel path accumulates it with atomics: measured cosines
            # 0.944-0.979 over seeds and runs, against 0.977-0.999 for every other matrix
            assert cos > 0.9 and abs(ratio - 1) < 0.15, (n, cos, ratio)
        else:
            assert cos > 0.95 and abs(ratio - 1) < 0.15, (n, cos, ratio)
