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
    """Gradients against an fp64 oracle on the same bf16-rounded inputs.  dA is an (H,) sum of
    ~B*L*64 products of both signs whose intra-chunk parts cancel (the gradient of a decay shift);
    the kernel keeps the cancelling sums at fp32 precision (exact diagonal blocks, two-term bf16
    operands elsewhere), so dA is held to 5e-2 like the per-element gradients."""
    ins = _inputs(B, L, H, 3, shift)
    xs = [t.clone().requires_grad_(True) for t in ins]
    y = K.ssd(*xs, 64)
    dy = torch.randn_like(y)
    (y.float() * dy.float()).sum().backward()
    rs = [t.detach().double().clone().requires_grad_(True) for t in ins]
    y2, _ = R.ssd_chunked(*rs, 64)
    (y2 * dy.double()).sum().backward()
    for name, a, r in zip(["dt", "A", "B", "C", "x"], xs, rs):
        assert torch.isfinite(a.grad).all(), name
        err = _rel(a.grad, r.grad)
        assert err < 5e-2, (name, err)
