"""CPU end-to-end checks of both model layouts, the parameter tree and training."""
import torch

from atomic_ai_hybrid_b200 import get_preset
from atomic_ai_hybrid_b200.models import HybridMoEModel, flax_path
from atomic_ai_hybrid_b200.training import compute_loss
from atomic_ai_hybrid_b200.training.trainer import Trainer


def _batch(cfg, B=2, L=128, seed=0):
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, cfg.vocab_size, (B, L + 1), generator=g)
    return {"input_ids": ids[:, :-1], "labels": ids[:, 1:]}


def test_reference_param_tree_names_and_dtypes():
    cfg = get_preset("reference_tiny")
    m = HybridMoEModel(cfg, compute_dtype=torch.float32)
    names = {flax_path(n): tuple(p.shape) for n, p in m.named_parameters()}
    d, dl, E = cfg.d_model, cfg.d_latent, cfg.e_routed
    # block 0 layer 0 has neither DAR nor intra parameters (no sources)
    assert not any(k.startswith("block_0/layer_0/dar") or k.startswith("block_0/layer_0/intra") for k in names)
    assert names["block_0/layer_1/intra/k_proj_1/kernel"] == (d, dl)
    assert names["block_1/layer_3/dar/k_proj/kernel"] == (d, dl)
    assert names["block_0/layer_0/sublayer/gdn2/q_conv_w"] == (d, 4)
    assert names["block_0/layer_0/sublayer/gdn2/decay_a"] == (cfg.n_heads,)
    assert names["block_0/layer_1/sublayer/mamba2/in_proj/kernel"] == (d, 2 * cfg.d_inner)
    assert names["block_0/layer_1/sublayer/mamba2/dt_proj/bias"] == (cfg.d_inner,)
    assert names["block_0/layer_1/sublayer/mamba2/A_log"] == (cfg.n_heads_ssm,)
    assert names["block_0/layer_2/sublayer/mla/W_kv_down/kernel"] == (d, dl)
    assert names["block_0/moe/routed_w1"] == (E, d, cfg.d_ff)
    assert names["block_0/moe/router"] == (d, E)
    assert names["block_0/moe/router_temp"] == ()
    assert names["block_0/moe/shared_w1/bias"] == (cfg.d_ff,)
    assert names["embed/embedding"] == (cfg.vocab_size, d)
    assert "final_norm/scale" in names


def test_forward_backward_both_layouts():
    for name in ("tiny", "reference_tiny"):
        cfg = get_preset(name)
        torch.manual_seed(0)
        m = HybridMoEModel(cfg, compute_dtype=torch.float32)
        loss, info = compute_loss(m, _batch(cfg))
        assert torch.isfinite(loss)
        loss.backward()
        assert all(torch.isfinite(p.grad).all() for p in m.parameters() if p.grad is not None)
        assert info["assignment_frac"].shape[1] == cfg.e_routed


def test_dar_is_dead_code():
    cfg = get_preset("reference_tiny")
    torch.manual_seed(0)
    m1 = HybridMoEModel(cfg, compute_dtype=torch.float32, compute_dar=False).eval()
    m2 = HybridMoEModel(cfg, compute_dtype=torch.float32, compute_dar=True).eval()
    m2.load_state_dict(m1.state_dict())
    b = _batch(cfg)
    with torch.no_grad():
        h1, _ = m1(b["input_ids"])
        h2, _ = m2(b["input_ids"])
    assert torch.equal(h1, h2)


def test_training_reduces_loss():
    cfg = get_preset("tiny", num_layers=2, layer_types=("mamba2", "gdn2"))
    torch.manual_seed(0)
    m = HybridMoEModel(cfg, compute_dtype=torch.float32)
    tr = Trainer(m, total_steps=50, optimizer="hybrid", compute_dtype=torch.float32, device=torch.device("cpu"))
    tr.opt.schedule.warmup = 2
    b = _batch(cfg, L=64)
    losses = [tr.train_step([b])["loss"].item() for _ in range(8)]
    assert losses[-1] < losses[0] - 0.5, losses


def test_activation_checkpointing_matches():
    """``remat=True`` recomputes every layer in the backward: same loss and gradients."""
    from atomic_ai_hybrid_b200.training.loss import compute_loss
    cfg = get_preset("tiny", num_layers=2, layer_types=("mamba2", "gdn2"), vocab_size=256, d_model=128,
                     n_heads=2, n_heads_ssm=2, d_ff=128, n_routed_experts=4, d_state=32)
    ids = torch.randint(0, cfg.vocab_size, (2, 65), generator=torch.Generator().manual_seed(3))
    batch = {"input_ids": ids[:, :-1], "labels": ids[:, 1:]}
    res = []
    for remat in (False, True):
        torch.manual_seed(0)
        m = HybridMoEModel(cfg, compute_dtype=torch.float32, remat=remat)
        loss, info = compute_loss(m, batch)
        loss.backward()
        res.append((loss.detach(), {n: p.grad.clone() for n, p in m.named_parameters() if p.grad is not None},
                    info["aux_loss"]))
    (l0, g0, a0), (l1, g1, a1) = res
    torch.testing.assert_close(l1, l0)
    torch.testing.assert_close(a1, a0)
    assert g0.keys() == g1.keys()
    for n in g0:
        torch.testing.assert_close(g1[n], g0[n], rtol=1e-5, atol=1e-7, msg=n)


def test_reference_preset_is_the_reference_training_config():
    """``reference`` = the ModelConfig the reference's train.py builds (`train.py:405-436`)."""
    c = get_preset("reference")
    assert (c.d_model, c.n_heads, c.d_latent, c.d_ff, c.num_experts, c.top_k) == (768, 6, 768, 4096, 8, 2)
    assert (c.num_layers, c.layers_per_block, c.vocab_size) == (24, 3, 128256)
    assert (c.router_aux_loss_coef, c.router_z_loss_coef, c.label_smoothing, c.router_noise_std) == \
        (0.03, 0.0003, 0.0, 0.1)
    assert c.deltanet_chunk_size == 256 and c.tie_embeddings and c.arch == "blockdar"
    assert c.layer_types[:6] == ("gdn2", "gdn2", "mla", "gdn2", "mamba2", "gdn2")
    assert c.layer_types[-3:] == ("gdn2", "gdn2", "gdn2") and c.layer_types.count("mla") == 4
