"""The chunked WY GDN-2 and chunked SSD oracles against token-serial ground truth
(the reference's validation method: chunked vs token-serial, fp64)."""
import torch
import torch.nn.functional as F

from atomic_ai_hybrid_b200.ops import reference as R


def _gdn_inputs(B=2, L=128, H=2, D=16, seed=0, dtype=torch.float64, strong_decay=False):
    g_ = torch.Generator().manual_seed(seed)
    q = F.normalize(torch.randn(B, L, H, D, generator=g_, dtype=dtype), dim=-1)
    k = F.normalize(torch.randn(B, L, H, D, generator=g_, dtype=dtype), dim=-1)
    v = torch.randn(B, L, H, D, generator=g_, dtype=dtype)
    g = -F.softplus(torch.randn(B, L, H, D, generator=g_, dtype=dtype)) * (20.0 if strong_decay else 1.0)
    b = torch.sigmoid(torch.randn(B, L, H, D, generator=g_, dtype=dtype))
    w = torch.sigmoid(torch.randn(B, L, H, D, generator=g_, dtype=dtype))
    return q, k, v, g, b, w


def test_gdn_chunked_matches_token_serial():
    q, k, v, g, b, w = _gdn_inputs()
    o1, h1 = R.gdn2_token_serial(q, k, v, g, b, w, 1.0)
    for C in (16, 32, 64):
        o2, h2 = R.gdn2_chunked(q, k, v, g, b, w, 1.0, C)
        assert torch.allclose(o1, o2, atol=1e-8, rtol=1e-7)
        assert torch.allclose(h1, h2, atol=1e-8, rtol=1e-7)


def test_gdn_chunked_scale_and_h0():
    q, k, v, g, b, w = _gdn_inputs(seed=1)
    h0 = torch.randn(2, 2, 16, 16, dtype=torch.float64)
    o1, h1 = R.gdn2_token_serial(q, k, v, g, b, w, 0.5, h0)
    o2, h2 = R.gdn2_chunked(q, k, v, g, b, w, 0.5, 32, h0)
    assert torch.allclose(o1, o2, atol=1e-8) and torch.allclose(h1, h2, atol=1e-8)


def test_gdn_strong_decay_close():
    # the +-20 clip on pairwise decay only floors terms below e^-20
    q, k, v, g, b, w = _gdn_inputs(seed=2, strong_decay=True)
    o1, _ = R.gdn2_token_serial(q, k, v, g, b, w, 1.0)
    o2, _ = R.gdn2_chunked(q, k, v, g, b, w, 1.0, 32)
    assert (o1 - o2).abs().max() < 1e-6


def test_ssd_chunked_matches_token_serial():
    g_ = torch.Generator().manual_seed(3)
    B, L, H, P, N = 2, 128, 3, 8, 16
    dt = F.softplus(torch.randn(B, L, H, P, generator=g_, dtype=torch.float64) - 2).clamp(1e-2, 1.0)
    A = -torch.exp(torch.rand(H, generator=g_, dtype=torch.float64))
    Bm = torch.randn(B, L, N, generator=g_, dtype=torch.float64)
    Cm = torch.randn(B, L, N, generator=g_, dtype=torch.float64)
    x = torch.randn(B, L, H, P, generator=g_, dtype=torch.float64)
    y1, s1 = R.ssd_token_serial(dt, A, Bm, Cm, x)
    for C in (16, 64):
        # the reference floors chunk-level decays at e^-20, visible at 1e-8 for C=64
        y2, s2 = R.ssd_chunked(dt, A, Bm, Cm, x, C)
        assert torch.allclose(y1, y2, atol=1e-6, rtol=1e-6)
        assert torch.allclose(s1, s2, atol=1e-6, rtol=1e-6)


def test_oracle_gradients_finite_and_agree():
    q, k, v, g, b, w = _gdn_inputs(B=1, L=64, H=1, D=8, seed=4)
    ins = [t.clone().requires_grad_(True) for t in (q, k, v, g, b, w)]
    o, _ = R.gdn2_chunked(*ins[:3], ins[3], ins[4], ins[5], 1.0, 16)
    do = torch.randn_like(o)
    gc = torch.autograd.grad((o * do).sum(), ins)
    ins2 = [t.clone().requires_grad_(True) for t in (q, k, v, g, b, w)]
    o2, _ = R.gdn2_token_serial(*ins2[:3], ins2[3], ins2[4], ins2[5], 1.0)
    gs = torch.autograd.grad((o2 * do).sum(), ins2)
    for a, c in zip(gc, gs):
        assert torch.isfinite(a).all()
        assert torch.allclose(a, c, atol=1e-7, rtol=1e-6)


def test_label_smoothed_ce_matches_formula():
    logits = torch.randn(10, 50, dtype=torch.float64)
    labels = torch.randint(0, 50, (10,))
    labels[3] = -100
    s, m = R.label_smoothed_ce(logits, labels, 0.1)
    lp = logits.log_softmax(-1)
    sp, sn = 0.9, 0.1 / 49
    tgt = torch.full_like(lp, sn)
    tgt.scatter_(1, labels.clamp(0)[:, None], sp)
    ref = -(tgt * lp).sum(-1)
    ref[3] = 0
    assert torch.allclose(s, ref.sum().float(), rtol=1e-5) and m.item() == 9
