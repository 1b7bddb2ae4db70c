"""The memory planner lays out the same stores as the trainer: its state bytes equal the
buffers a real trainer allocates for the same model and layout (tiny model, CPU)."""
import torch

from atomic_ai_hybrid_b200 import get_preset
from atomic_ai_hybrid_b200.models import HybridMoEModel
from atomic_ai_hybrid_b200.utils import memplan


def _cfg():
    return get_preset("tiny", num_layers=2, layer_types=("mamba2", "gdn2"), vocab_size=512, d_model=128, n_heads=2,
                      n_heads_ssm=2, d_ff=128, n_routed_experts=4, d_state=32)


def test_state_bytes_match_trainer_buffers():
    from atomic_ai_hybrid_b200.training.trainer import Trainer
    cfg = _cfg()
    torch.manual_seed(0)
    tr = Trainer(HybridMoEModel(cfg, compute_dtype=torch.bfloat16), total_steps=10, optimizer="adamw",
                 compute_dtype=torch.bfloat16, device=torch.device("cpu"))
    st, opt = tr.store, tr.opt
    real = {"master": st.master.numel() * 4, "grad": st.grad.numel() * 4,
            "compute": st.compute.numel() * st.compute.element_size(),
            "optimizer": (opt.m.numel() + opt.v.numel()) * 4}
    got = memplan.plan(cfg, world=1, micro_batch=1, seq_len=64)
    for k, v in real.items():
        assert abs(got["state_gb"][k] * 1e9 - v) <= 0.01e9, (k, got["state_gb"][k], v)
    assert got["params_replicated"] == sum(p.numel() for p in tr.model.parameters())


def test_layouts_divide_state_and_tokens():
    cfg = _cfg()
    one = memplan.plan(cfg, world=1, micro_batch=2, seq_len=256)
    dp4 = memplan.plan(cfg, world=4, micro_batch=2, seq_len=256)
    # sharded data parallelism: master and moments split four ways, gradients and compute copy do not
    assert dp4["state_gb"]["grad"] == one["state_gb"]["grad"]
    assert dp4["state_gb"]["optimizer"] <= one["state_gb"]["optimizer"] / 4 + 0.01
    ep2 = memplan.plan(cfg, world=2, ep=2, micro_batch=2, seq_len=256)
    assert ep2["params_local"] > 0 and ep2["params_local"] + ep2["params_replicated"] < one["params_replicated"]
    tp2 = memplan.plan(cfg, world=2, tp=2, micro_batch=2, seq_len=256)
    assert tp2["params_local"] > 0  # the head-split pieces
    act = memplan.activation_bytes
    assert act(cfg, 2, 256, 2, tp=2) == act(cfg, 2, 256, 2) / 2 == act(cfg, 2, 256, 2, cp=2)
    assert act(cfg, 2, 256, 2, remat=True) < act(cfg, 2, 256, 2)
    assert act(cfg, 2, 256, 1, in_flight=3) == 3 * act(cfg, 2, 256, 1)
    pp2 = memplan.plan(cfg, world=2, pp=2, micro_batch=2, seq_len=256, accum_steps=4)
    assert pp2["layout"]["stage"] in (0, 1) and pp2["params_replicated"] < one["params_replicated"]


def test_benchmark_config_plans():
    """The 1-GPU benchmark layout fits (it runs); the long-context configuration's state
    does not fit with fp32 gradients for its 10 B rank-local parameters, and does with
    16-bit ones."""
    one = memplan.plan(get_preset("hybrid_1b"), world=1, micro_batch=4, seq_len=4096)
    assert one["fits"] and abs(one["total_gb"] - 169.8) < 1.0
    long32 = memplan.plan(get_preset("hybrid_long"), world=8, tp=8, ep=8, micro_batch=1, seq_len=32768, remat=True)
    assert not long32["fits"] and long32["state_total_gb"] > long32["hbm_gb"]
    long16 = memplan.plan(get_preset("hybrid_long"), world=8, tp=8, ep=8, micro_batch=1, seq_len=32768, remat=True,
                          local_grad_bytes=2)
    assert long16["fits"]


def test_run_files_for_eight_gpus():
    """The 8-GPU run files fit as written (configuration 5 with bf16 gradient accumulators for
    its 9.7 B expert weights per GPU; with fp32 ones it does not: ``test_benchmark_config_plans``).
    The alternative layout with the rank-local AdamW moments in pinned host memory takes 82 GB
    per rank and 657 GB per node: it does not fit a 512 GB node."""
    import os
    root = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "atomic_ai_hybrid_b200",
                        "configs")
    for name, fits in (("config3_hybrid_1b.yaml", True), ("config4_hybrid_7b_ep8.yaml", True),
                       ("config5_hybrid_long_tp8.yaml", True)):
        out = memplan.main(["--config", os.path.join(root, name), "--world", "8", "--host-ram-gb", "2048"])
        assert out["fits"] is fits, (name, out)
    c5 = memplan.main(["--config", os.path.join(root, "config5_hybrid_long_tp8.yaml"), "--world", "8"])
    assert c5["fits"] and c5["host_pinned_gb_per_rank"] == 0 and c5["total_gb"] < c5["hbm_gb"]
    c5 = memplan.main(["--config", os.path.join(root, "config5_hybrid_long_tp8.yaml"), "--world", "8",
                       "--host-ram-gb", "512", "--offload-local-moments"])
    assert not c5["fits"] and not c5["host_fits"] and c5["total_gb"] <= c5["hbm_gb"]
    assert abs(c5["host_pinned_gb_per_rank"] - 82.1) < 1.0
    assert abs(c5["host_pinned_gb_per_node"] - 8 * c5["host_pinned_gb_per_rank"]) < 0.1


def test_host_pinned_accounting():
    """Moments kept on the device count 8 bytes per rank-local parameter in HBM and none on
    the host; staged ones move exactly those bytes to the host figures."""
    cfg = get_preset("hybrid_1b")
    kw = dict(world=2, ep=2, micro_batch=1, seq_len=256)
    dev = memplan.plan(cfg, **kw)
    host = memplan.plan(cfg, local_moments_on_host=True, host_ram_gb=1e4, **kw)
    assert dev["host_pinned_gb_per_rank"] == 0 and dev["host_fits"]
    moved = dev["state_gb"]["optimizer"] - host["state_gb"]["optimizer"]
    assert moved > 1.0 and abs(moved - host["host_pinned_gb_per_rank"]) < 0.02
    assert abs(host["host_pinned_gb_per_node"] - 2 * host["host_pinned_gb_per_rank"]) < 0.02
    tight = memplan.plan(cfg, local_moments_on_host=True, host_ram_gb=host["host_pinned_gb_per_node"], **kw)
    assert not tight["host_fits"] and not tight["fits"]


def test_offloaded_moments_train_like_device_moments(tmp_path):
    """``offload_moments``: the same updates and moments as device-resident ones, no fused
    kernel, and the moments save to / restore from checkpoints."""
    from atomic_ai_hybrid_b200.ckpt.manager import CheckpointManager
    from atomic_ai_hybrid_b200.optim import FlatParamStore, HybridOptimizer, grad_scale_of, label_adamw_only
    cfg = _cfg()
    outs = []
    for offload in (False, True):
        torch.manual_seed(0)
        m = HybridMoEModel(cfg, compute_dtype=torch.float32)
        st = FlatParamStore(m, label_adamw_only, grad_scale_of, 1, 0, compute_dtype=torch.float32,
                            device=torch.device("cpu"))
        opt = HybridOptimizer(st, 10, offload_moments=offload)
        opt.schedule.warmup = 1
        g = torch.Generator().manual_seed(3)
        for _ in range(3):
            st.grad.copy_(torch.randn(st.grad.shape, generator=g) * 1e-3)
            opt.step(1)
        assert opt.uses_kernels() is False
        outs.append((st.master.clone(), opt.m.clone(), opt.v.clone()))
    for a, b in zip(*outs):
        assert torch.equal(a, b)

    class _T:  # the two attributes a checkpoint reads
        pass
    t = _T()
    t.store, t.opt = st, opt
    CheckpointManager(str(tmp_path), "latest").save(3, t, asynchronous=False)
    m2 = opt.m.clone()
    opt.m.zero_()
    opt.v.zero_()
    CheckpointManager(str(tmp_path), "latest").restore(3, t)
    assert torch.equal(opt.m, m2)
