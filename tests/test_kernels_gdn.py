"""sm_100a GDN-2 kernels against the fp32 chunked-WY oracle (and token-serial truth)."""
import pytest
import torch
import torch.nn.functional as F

from atomic_ai_hybrid_b200.ops import kernels as K
from atomic_ai_hybrid_b200.ops import reference as R

pytestmark = pytest.mark.gpu
dev = "cuda"


def _inputs(B, L, H, seed, decay=1.0):
    g_ = torch.Generator(device=dev).manual_seed(seed)
    D = 128
    q = F.normalize(torch.randn(B, L, H, D, generator=g_, device=dev), dim=-1)
    k = F.normalize(torch.randn(B, L, H, D, generator=g_, device=dev), dim=-1)
    v = torch.randn(B, L, H, D, generator=g_, device=dev)
    g = -F.softplus(torch.randn(B, L, H, D, generator=g_, device=dev)) * decay
    b = torch.sigmoid(torch.randn(B, L, H, D, generator=g_, device=dev))
    w = torch.sigmoid(torch.randn(B, L, H, D, generator=g_, device=dev))
    bf = torch.bfloat16
    return q.to(bf), k.to(bf), v.to(bf), g, b.to(bf), w.to(bf)


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("B,L,H,decay", [(1, 64, 1, 1.0), (2, 256, 3, 1.0), (1, 512, 2, 0.05), (1, 192, 2, 8.0)])
def test_gdn_forward(B, L, H, decay):
    q, k, v, g, b, w = _inputs(B, L, H, 0, decay)
    o = K.gdn2(q, k, v, w, b, g, 1.0, 64)
    o_ref, _ = R.gdn2_chunked(q.float(), k.float(), v.float(), g, b.float(), w.float(), 1.0, 64)
    assert torch.isfinite(o).all()
    assert _rel(o, o_ref) < 2e-2, _rel(o, o_ref)


def test_gdn_forward_scale_matches_token_serial():
    q, k, v, g, b, w = _inputs(1, 128, 2, 1)
    o = K.gdn2(q, k, v, w, b, g, 0.5, 64)
    o_ref, _ = R.gdn2_token_serial(q.double(), k.double(), v.double(), g.double(), b.double(), w.double(), 0.5)
    assert _rel(o, o_ref) < 2e-2


# (5, 128, 16): 80 (batch, head) pairs keep the whole state in one CTA each; the smaller shapes split
# the value columns over two CTAs (the state kernels' two launch forms)
@pytest.mark.parametrize("B,L,H,decay", [(1, 128, 1, 1.0), (2, 256, 2, 0.1), (1, 192, 1, 4.0), (5, 128, 16, 1.0)])
def test_gdn_backward(B, L, H, decay):
    ins = _inputs(B, L, H, 2, decay)
    xs = [t.clone().requires_grad_(True) for t in ins]
    o = K.gdn2(xs[0], xs[1], xs[2], xs[5], xs[4], xs[3], 1.0, 64)
    do = torch.randn_like(o)
    (o.float() * do.float()).sum().backward()
    rs = [t.detach().float().clone().requires_grad_(True) for t in ins]
    o2, _ = R.gdn2_chunked(rs[0], rs[1], rs[2], rs[3], rs[4], rs[5], 1.0, 64)
    (o2 * do.float()).sum().backward()
    for name, a, r in zip("qkvgbw", xs, rs):
        assert torch.isfinite(a.grad).all(), name
        err = _rel(a.grad, r.grad)
        assert err < 5e-2, (name, err)


def test_gdn_production_shape_forward_backward():
    """The op-benchmark shape per sequence (T = 4096, H = 16, D = 128; two sequences): 64 chunks
    per head, so index arithmetic at long T and the full state recurrence are checked against
    the fp32 chunked oracle."""
    B, L, H = 2, 4096, 16
    ins = _inputs(B, L, H, 5)
    xs = [t.clone().requires_grad_(True) for t in ins]
    o = K.gdn2(xs[0], xs[1], xs[2], xs[5], xs[4], xs[3], 1.0, 64)
    do = torch.randn_like(o)
    (o.float() * do.float()).sum().backward()
    rs = [t.detach().float().clone().requires_grad_(True) for t in ins]
    o2, _ = R.gdn2_chunked(rs[0], rs[1], rs[2], rs[3], rs[4], rs[5], 1.0, 64, checkpoint_chunks=True)
    assert _rel(o, o2) < 2e-2, _rel(o, o2)
    (o2 * do.float()).sum().backward()
    for name, a, r in zip("qkvgbw", xs, rs):
        assert torch.isfinite(a.grad).all(), name
        err = _rel(a.grad, r.grad)
        assert err < 5e-2, (name, err)


@pytest.mark.parametrize("recompute", [False, True])
def test_gdn_initial_state_and_final_state(recompute, monkeypatch):
    """``h0`` in and the final state out, both with gradients (saved-intermediates and
    recompute backward paths), against the fp32 chunked oracle started from the same state;
    the loss also reads the final state, so its gradient enters the reverse recurrence."""
    monkeypatch.setattr(K, "SCAN_RECOMPUTE", recompute)
    B, L, H = 2, 256, 2
    ins = _inputs(B, L, H, 7)
    g_ = torch.Generator(device=dev).manual_seed(8)
    h0 = (torch.randn(B, H, 128, 128, generator=g_, device=dev) * 0.1)
    xs = [t.clone().requires_grad_(True) for t in ins]
    hx = h0.clone().requires_grad_(True)
    o, hf = K.gdn2(xs[0], xs[1], xs[2], xs[5], xs[4], xs[3], 1.0, 64, h0=hx, return_final=True)
    do = torch.randn_like(o)
    dhf = torch.randn_like(hf) * 0.1
    ((o.float() * do.float()).sum() + (hf * dhf).sum()).backward()
    rs = [t.detach().float().clone().requires_grad_(True) for t in ins]
    hr = h0.clone().requires_grad_(True)
    o2, hf2 = R.gdn2_chunked(rs[0], rs[1], rs[2], rs[3], rs[4], rs[5], 1.0, 64, h0=hr)
    ((o2 * do.float()).sum() + (hf2 * dhf).sum()).backward()
    assert _rel(o, o2) < 2e-2, _rel(o, o2)
    assert _rel(hf, hf2) < 2e-2, _rel(hf, hf2)
    for name, a, r in zip("qkvgbw", xs, rs):
        assert torch.isfinite(a.grad).all(), name
        assert _rel(a.grad, r.grad) < 5e-2, (name, _rel(a.grad, r.grad))
    assert _rel(hx.grad, hr.grad) < 3e-2, _rel(hx.grad, hr.grad)
