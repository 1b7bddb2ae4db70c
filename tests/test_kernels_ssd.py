"""sm_100a Mamba2 SSD kernels against the fp32 chunked oracle with the reference's clips."""
import math

import pytest
import torch
import torch.nn.functional as F

from atomic_ai_hybrid_b200.ops import kernels as K
from atomic_ai_hybrid_b200.ops import reference as R

pytestmark = pytest.mark.gpu
dev = "cuda"


def _inputs(B, L, H, seed, dt_shift=-4.0):
    g_ = torch.Generator(device=dev).manual_seed(seed)
    P, N = 64, 128
    x = torch.randn(B, L, H, P, generator=g_, device=dev)
    dt = F.softplus(torch.randn(B, L, H, P, generator=g_, device=dev) + dt_shift).clamp(1e-2, 1.0)
    A = -torch.exp(torch.rand(H, generator=g_, device=dev) * math.log(16.0))
    Bm = torch.randn(B, L, N, generator=g_, device=dev) / math.sqrt(N)
    Cm = torch.randn(B, L, N, generator=g_, device=dev) / math.sqrt(N)
    bf = torch.bfloat16
    return dt.to(bf), A, Bm.to(bf), Cm.to(bf), x.to(bf)


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("B,L,H,shift", [(1, 64, 1, -4.0), (2, 256, 3, -4.0), (1, 320, 2, 0.0), (1, 128, 2, 2.0)])
def test_ssd_forward(B, L, H, shift):
    dt, A, Bm, Cm, x = _inputs(B, L, H, 0, shift)
    y = K.ssd(dt, A, Bm, Cm, x, 64)
    y_ref, _ = R.ssd_chunked(dt.float(), A, Bm.float(), Cm.float(), x.float(), 64)
    assert torch.isfinite(y).all()
    assert _rel(y, y_ref) < 2e-2, _rel(y, y_ref)


@pytest.mark.parametrize("B,L,H,shift", [(1, 128, 1, -4.0), (2, 192, 2, -1.0), (1, 128, 2, 2.0), (2, 256, 3, -1.0)])
def test_ssd_backward(B, L, H, shift):
    """Gradients against an fp64 oracle on the same bf16-rounded inputs (per-element gradients
    to 5e-2 relative).  dA[h] = sum_{b,t,p} g * dt over ~B*L*64 terms of both signs, g the
    reverse cumulative sum of the decay gradient; for some dy a head's sum nearly cancels, so it is
    checked per head against 5e-2 of its value plus 1e-3 of sum |g dt| (g from the oracle's own
    dt / x gradients: ddt = g A + d(dBx) x, dx = d(dBx) dt) -- a missed or doubled term is off by
    a sizeable part of that sum."""
    _check_backward(B, L, H, shift, seed=3)


def _check_backward(B, L, H, shift, seed):
    ins = _inputs(B, L, H, seed, shift)
    xs = [t.clone().requires_grad_(True) for t in ins]
    y = K.ssd(*xs, 64)
    dy = torch.randn(y.shape, generator=torch.Generator(device=dev).manual_seed(seed + 100), device=dev).to(y.dtype)
    (y.float() * dy.float()).sum().backward()
    rs = [t.detach().double().clone().requires_grad_(True) for t in ins]
    y2, _ = R.ssd_chunked(*rs, 64)
    (y2 * dy.double()).sum().backward()
    for name, a, r in zip(["dt", "A", "B", "C", "x"], xs, rs):
        assert torch.isfinite(a.grad).all(), name
        if name == "A":
            dt64, x64, A64 = rs[0].detach(), rs[4].detach(), rs[1].detach()
            g_dt = (rs[0].grad * dt64 - rs[4].grad * x64) / A64.view(1, 1, -1, 1)  # g * dt per element
            scale = g_dt.abs().sum(dim=(0, 1, 3))
            err = (a.grad.double() - r.grad).abs()
            bound = 5e-2 * r.grad.abs() + 1e-3 * scale
            assert (err <= bound).all(), (name, err.tolist(), bound.tolist())
        else:
            err = _rel(a.grad, r.grad)
            assert err < 5e-2, (name, err)


def test_ssd_production_shape_forward_backward():
    """The op-benchmark shape per sequence (T = 4096, H = 32, P = 64, N = 128): 64 chunks per head,
    all four head groups of the chunk backward, against the fp64 oracle."""
    _check_backward(1, 4096, 32, -4.0, seed=5)


@pytest.mark.parametrize("recompute", [False, True])
def test_ssd_initial_state_and_final_state(recompute, monkeypatch):
    """``state0`` in and the final state out, both with gradients (saved-states and
    recompute backward paths), against the fp64 oracle started from the same state; the loss
    also reads the final state, so its gradient enters the reverse recurrence."""
    monkeypatch.setattr(K, "SCAN_RECOMPUTE", recompute)
    B, L, H = 2, 256, 3
    ins = _inputs(B, L, H, 11, -1.0)
    g_ = torch.Generator(device=dev).manual_seed(12)
    s0 = torch.randn(B, H, 64, 128, generator=g_, device=dev) * 0.5
    xs = [t.clone().requires_grad_(True) for t in ins]
    sx = s0.clone().requires_grad_(True)
    y, sf = K.ssd(*xs, 64, state0=sx, return_final=True)
    dy = torch.randn(y.shape, generator=g_, device=dev).to(y.dtype)
    dsf = torch.randn(sf.shape, generator=g_, device=dev) * 0.1
    ((y.float() * dy.float()).sum() + (sf * dsf).sum()).backward()
    rs = [t.detach().double().clone().requires_grad_(True) for t in ins]
    sr = s0.double().clone().requires_grad_(True)
    y2, sf2 = R.ssd_chunked(*rs, 64, state0=sr)
    ((y2 * dy.double()).sum() + (sf2 * dsf.double()).sum()).backward()
    assert _rel(y, y2) < 2e-2, _rel(y, y2)
    assert _rel(sf, sf2) < 2e-2, _rel(sf, sf2)
    for name, a, r in zip(["dt", "A", "B", "C", "x"], xs, rs):
        assert torch.isfinite(a.grad).all(), name
        assert _rel(a.grad, r.grad) < 5e-2, (name, _rel(a.grad, r.grad))
    assert _rel(sx.grad, sr.grad) < 2e-2, _rel(sx.grad, sr.grad)
