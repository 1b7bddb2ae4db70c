"""Dense projections on the tcgen05 GEMM (single CTA below 256 rows, CTA pairs above) against
PyTorch fp32: forward with bias, the accumulated input gradient and the fp32 weight-gradient
accumulation, and the multi-projection autograd op."""
import pytest
import torch

from atomic_ai_hybrid_b200.ops import kernels as KN
from atomic_ai_hybrid_b200.ops._ext import ext

pytestmark = pytest.mark.gpu
dev = "cuda"


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("M,K,N", [(128, 64, 32), (1000, 256, 128), (4096, 2048, 2048), (16384, 2048, 4096)])
def test_dense_fwd_dgrad_wgrad(M, K, N):
    ext().gemm_error_reset()
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
    W = (torch.randn(K, N, device=dev, generator=g) / K ** 0.5).to(torch.bfloat16)
    b = torch.randn(N, device=dev, generator=g).to(torch.bfloat16)
    y = ext().dense_fwd(x, W, b)
    ref = x.float() @ W.float() + b.float()
    assert _rel(y, ref) < 1e-2, _rel(y, ref)
    dy = torch.randn(M, N, device=dev, generator=g).to(torch.bfloat16)
    if N % 64 == 0:
        dx = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
        dx0 = dx.clone()
        ext().dense_dgrad(dy, W, dx, True)
        ref = dx0.float() + dy.float() @ W.float().t()
        assert _rel(dx, ref) < 1e-2, _rel(dx, ref)
    if K % 128 == 0:
        acc = torch.randn(K, N, device=dev, generator=g)
        acc0 = acc.clone()
        ext().dense_wgrad(x, dy, acc)
        ref = acc0 + x.float().t() @ dy.float()
        assert _rel(acc, ref) < 1e-3, _rel(acc, ref)
    torch.cuda.synchronize()
    assert KN.gemm_error() == 0


def test_linear_multi_matches_fp32():
    """Three projections of one input (with and without bias) through autograd: outputs, the
    input gradient summed over the projections, and weight / bias gradients."""
    g = torch.Generator(device=dev).manual_seed(1)
    M, K = 600, 512
    x = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16).requires_grad_(True)
    shapes = [(K, 512), (K, 128), (K, 1024)]
    ws = [(torch.randn(*s, device=dev, generator=g) / K ** 0.5).to(torch.bfloat16).requires_grad_(True) for s in shapes]
    bs = [None, torch.randn(128, device=dev, generator=g).to(torch.bfloat16).requires_grad_(True), None]
    outs = KN.linear_multi(x, list(zip(ws, bs)))
    dys = [torch.randn_like(o) for o in outs]
    sum((o.float() * d.float()).sum() for o, d in zip(outs, dys)).backward()
    xr = x.detach().float().requires_grad_(True)
    wr = [w.detach().float().requires_grad_(True) for w in ws]
    br = [b.detach().float().requires_grad_(True) if b is not None else None for b in bs]
    refs = [xr @ w + (b if b is not None else 0) for w, b in zip(wr, br)]
    sum((o * d.float()).sum() for o, d in zip(refs, dys)).backward()
    for o, r in zip(outs, refs):
        assert _rel(o, r) < 1e-2
    assert _rel(x.grad, xr.grad) < 1e-2, _rel(x.grad, xr.grad)
    for w, r in zip(ws, wr):
        assert _rel(w.grad, r.grad) < 1e-2, _rel(w.grad, r.grad)
    assert _rel(bs[1].grad, br[1].grad) < 1e-2


def test_dense_strided_operands():
    """Column slices of wider row-major buffers (as a fused kernel's outputs are handed out)
    enter the GEMMs and the bias-gradient kernel as views, without copies, and give the same
    results as contiguous operands."""
    from atomic_ai_hybrid_b200.ops.kernels import bias_grad
    g = torch.Generator(device=dev).manual_seed(5)
    M, K, N = 1000, 512, 256
    xw = torch.randn(M, 3 * K, device=dev, generator=g).to(torch.bfloat16)
    dyw = torch.randn(M, 2 * N, device=dev, generator=g).to(torch.bfloat16)
    x, dy = xw[:, K:2 * K], dyw[:, N:]
    assert not x.is_contiguous() and not dy.is_contiguous()
    W = (torch.randn(K, N, device=dev, generator=g) / K ** 0.5).to(torch.bfloat16)
    y = ext().dense_fwd(x, W, None)
    assert torch.equal(y, ext().dense_fwd(x.contiguous(), W, None))
    dx = torch.empty(M, K, device=dev, dtype=torch.bfloat16)
    ext().dense_dgrad(dy, W, dx, False)
    dx2 = torch.empty_like(dx)
    ext().dense_dgrad(dy.contiguous(), W, dx2, False)
    assert torch.equal(dx, dx2)
    a1, a2 = torch.zeros(K, N, device=dev), torch.zeros(K, N, device=dev)
    ext().dense_wgrad(x, dy, a1)
    ext().dense_wgrad(x.contiguous(), dy.contiguous(), a2)
    assert torch.equal(a1, a2)
    b = torch.zeros(N, device=dev, dtype=torch.bfloat16)
    b._ahb_grad_acc = torch.zeros(N, device=dev)
    assert bias_grad(b, dy) is None
    torch.testing.assert_close(b._ahb_grad_acc, dy.float().sum(0), rtol=1e-3, atol=1e-2)
