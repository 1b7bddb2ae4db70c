"""sm_100a elementwise kernels against plain-PyTorch fp32 references."""
import pytest
import torch

from atomic_ai_hybrid_b200.ops import kernels as K
from atomic_ai_hybrid_b200.ops import reference as R

pytestmark = pytest.mark.gpu
dev = "cuda"


@pytest.mark.parametrize("D", [256, 768, 2048, 4096])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_rmsnorm_fwd_bwd(D, dtype):
    torch.manual_seed(0)
    x = torch.randn(37, 5, D, device=dev, dtype=dtype, requires_grad=True)
    s = (1 + 0.1 * torch.randn(D, device=dev)).requires_grad_(True)
    y = K.rmsnorm(x, s, 1e-6)
    dy = torch.randn_like(y)
    (y.float() * dy.float()).sum().backward()
    x2 = x.detach().float().requires_grad_(True)
    s2 = s.detach().clone().requires_grad_(True)
    y2 = R.rmsnorm(x2, s2, 1e-6)
    (y2 * dy.float()).sum().backward()
    tol = 2e-2 if dtype == torch.bfloat16 else 1e-4
    torch.testing.assert_close(y.float(), y2, atol=tol, rtol=tol)
    torch.testing.assert_close(x.grad.float(), x2.grad, atol=tol, rtol=tol)
    torch.testing.assert_close(s.grad, s2.grad, atol=tol * 40, rtol=tol)


@pytest.mark.parametrize("silu,clip", [(True, 0.0), (True, 0.5), (False, 0.0)])
def test_conv1d_fwd_bwd(silu, clip):
    torch.manual_seed(1)
    B, L, C = 2, 77, 64
    big = torch.randn(B, L, 2 * C, device=dev, dtype=torch.float32)
    x = big[..., :C].detach().requires_grad_(False)
    xr = x.clone().requires_grad_(True)
    w = (0.3 * torch.randn(C, 4, device=dev)).requires_grad_(True)
    b = (0.1 * torch.randn(C, device=dev)).requires_grad_(True)
    xk = x.clone().requires_grad_(True)
    y = K.conv1d(xk, w, b, silu, clip if clip else None)
    w2 = w.detach().clone().requires_grad_(True)
    b2 = b.detach().clone().requires_grad_(True)
    y2 = R.causal_conv1d(xr, w2, b2, silu)
    if clip:
        y2 = y2.clamp(-clip, clip)
    torch.testing.assert_close(y, y2, atol=1e-4, rtol=1e-4)
    dy = torch.randn_like(y)
    (y * dy).sum().backward()
    (y2 * dy).sum().backward()
    torch.testing.assert_close(xk.grad, xr.grad, atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(w.grad, w2.grad, atol=1e-3, rtol=1e-3)
    torch.testing.assert_close(b.grad, b2.grad, atol=1e-3, rtol=1e-3)


def test_conv1d_strided_input_bf16():
    torch.manual_seed(2)
    xz = torch.randn(2, 64, 256, device=dev, dtype=torch.bfloat16)
    x = xz[..., :128]
    w = 0.3 * torch.randn(128, 4, device=dev, dtype=torch.bfloat16)
    y = K.conv1d(x, w, None, True)
    y2 = R.causal_conv1d(x.float(), w.float(), None, True)
    torch.testing.assert_close(y.float(), y2, atol=2e-2, rtol=2e-2)


def test_sanitize_and_embedding():
    x = torch.tensor([1.0, float("nan"), float("inf"), -float("inf"), 5e3, -2.0], device=dev)
    torch.testing.assert_close(K.sanitize(x, 1e3), R.sanitize(x, 1e3))
    emb = torch.randn(100, 64, device=dev, requires_grad=True)
    ids = torch.randint(0, 100, (3, 7), device=dev)
    out = K.embedding(ids, emb, torch.float32)
    torch.testing.assert_close(out, emb.detach()[ids])
    out.sum().backward()
    ref = torch.zeros_like(emb)
    ref.index_add_(0, ids.reshape(-1), torch.ones(21, 64, device=dev))
    torch.testing.assert_close(emb.grad, ref)


@pytest.mark.parametrize("silu,clip,wdt", [(True, 0.0, torch.bfloat16), (True, 50.0, torch.float32),
                                           (False, 0.0, torch.bfloat16)])
def test_conv1d_streaming_bf16_fwd_bwd(silu, clip, wdt):
    """bf16 activations with C % 128 == 0 take the streaming kernels (spans of 64 steps)."""
    torch.manual_seed(3)
    B, L, C = 2, 203, 256
    xz = (torch.randn(B, L, 2 * C, device=dev) * 3).to(torch.bfloat16)
    x = xz[..., C:]  # strided rows
    w = (0.5 * torch.randn(C, 4, device=dev)).to(wdt).requires_grad_(True)
    b = (0.1 * torch.randn(C, device=dev)).requires_grad_(True)
    xk = xz.clone().requires_grad_(True)
    y = K.conv1d(xk[..., C:], w, b, silu, clip if clip else None)
    xr = x.float().clone().requires_grad_(True)
    w2 = w.detach().float().clone().requires_grad_(True)
    b2 = b.detach().clone().requires_grad_(True)
    y2 = R.causal_conv1d(xr, w2, b2, silu)
    if clip:
        y2 = y2.clamp(-clip, clip)
    torch.testing.assert_close(y.float(), y2, atol=3e-2, rtol=2e-2)
    dy = torch.randn(B, L, C, device=dev).to(torch.bfloat16)
    y.backward(dy)
    y2.backward(dy.float())
    torch.testing.assert_close(xk.grad[..., C:].float(), xr.grad, atol=3e-2, rtol=2e-2)
    assert not xk.grad[..., :C].any()
    torch.testing.assert_close(w.grad.float(), w2.grad, atol=0.5, rtol=2e-2)
    torch.testing.assert_close(b.grad, b2.grad, atol=0.5, rtol=2e-2)
