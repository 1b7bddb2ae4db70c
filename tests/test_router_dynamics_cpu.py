"""Synthetic single-layer MoE dynamics (the reference's router tests,
`train_setup.py:67-122`): with every learning rate at zero, the expert-bias hook
alone must pull a router that prefers one expert back towards balance, and the
router-temperature hook must decay the temperature towards its initial value."""
import torch
import torch.nn.functional as F

from atomic_ai_hybrid_b200 import get_preset
from atomic_ai_hybrid_b200.models import HybridMoEModel
from atomic_ai_hybrid_b200.training.trainer import Trainer


def _setup():
    cfg = get_preset("tiny", num_layers=1, layer_types=("gdn2",), vocab_size=256, d_model=128, n_heads=2,
                     n_heads_ssm=2, d_ff=128, n_routed_experts=4, top_k=1, d_state=32)
    torch.manual_seed(0)
    m = HybridMoEModel(cfg, compute_dtype=torch.float32)
    ids = torch.randint(0, cfg.vocab_size, (4, 65), generator=torch.Generator().manual_seed(2))
    seen = {}

    def grab(mod, args):
        seen.setdefault("x", args[0].detach())

    h = m.layer_0.moe.register_forward_pre_hook(grab)
    with torch.no_grad():
        m(ids[:, :-1])
    h.remove()
    x = seen["x"].reshape(-1, cfg.d_model)
    dirn = F.normalize(x.mean(0), dim=0)
    with torch.no_grad():
        r = m.layer_0.moe.router
        r[:, 0] = (0.6 * dirn + 0.4 * F.normalize(r[:, 0], dim=0)) * r[:, 0].norm()
    tr = Trainer(m, total_steps=100, optimizer="adamw", compute_dtype=torch.float32, device=torch.device("cpu"))
    tr.opt.base = {k: 0.0 for k in tr.opt.base}
    return m, tr, {"input_ids": ids[:, :-1], "labels": ids[:, 1:]}


def _frac(tr, batch):
    tr.micro_step(batch)
    f = tr._frac_sum.clone() / tr._n_micro
    return f[0]


def test_expert_bias_hook_rebalances_routing():
    m, tr, batch = _setup()
    first = None
    for step in range(60):
        f = _frac(tr, batch)
        if first is None:
            first = f.clone()
        tr.apply(1)
    last = _frac(tr, batch)
    assert first[0] > 0.35, first  # the skewed router prefers expert 0
    assert last.std() < 0.7 * first.std(), (first, last)
    bias = m.layer_0.moe.expert_bias.detach()
    assert bias[0] < 0 and bias[1:].min() > bias[0], bias


def test_router_temperature_decays_towards_init():
    m, tr, batch = _setup()
    with torch.no_grad():
        tr.store.master_view(tr.store.by_name["layer_0.moe.router_temp"]).fill_(14.0)
    for _ in range(20):
        tr.micro_step(batch)
        tr.apply(1)
    t = float(m.layer_0.moe.router_temp.detach())
    # t <- t - 0.02 (t - 10) per step, with no gradient step (zero learning rates)
    assert abs(t - (10.0 + 4.0 * 0.98 ** 20)) < 1e-3, t
