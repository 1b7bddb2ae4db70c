"""tcgen05 grouped GEMM and the MoE dispatch/combine kernels against PyTorch fp32."""
import pytest
import torch

from atomic_ai_hybrid_b200.ops import kernels as KN
from atomic_ai_hybrid_b200.ops import reference as R
from atomic_ai_hybrid_b200.ops._ext import ext

pytestmark = pytest.mark.gpu
dev = "cuda"


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("M,K,N", [(128, 64, 256), (256, 128, 256), (1024, 2048, 512), (384, 320, 768)])
def test_gemm_dense(M, K, N):
    ext().gemm_error_reset()
    torch.manual_seed(0)
    a = torch.randn(M, K, device=dev, dtype=torch.bfloat16)
    b = torch.randn(N, K, device=dev, dtype=torch.bfloat16)
    c = ext().gemm_dense(a, b)
    torch.cuda.synchronize()
    assert KN.gemm_error() == 0
    ref = a.float() @ b.float().t()
    assert _rel(c, ref) < 1e-2, _rel(c, ref)


@pytest.mark.parametrize("M,K,N", [(256, 64, 256), (512, 2048, 512), (1000, 320, 768), (4096, 2048, 2048)])
def test_gemm_dense_cta_pair(M, K, N):
    """The CTA-pair kernel (cta_group::2, 256 x 256 tiles over two SMs) against fp32, including a
    last tile that runs past M (rows read as zeros, not stored)."""
    ext().gemm_error_reset()
    torch.manual_seed(2)
    a = torch.randn(M, K, device=dev, dtype=torch.bfloat16)
    b = torch.randn(N, K, device=dev, dtype=torch.bfloat16)
    c = ext().gemm_dense(a, b, pair=True)
    torch.cuda.synchronize()
    assert KN.gemm_error() == 0
    ref = a.float() @ b.float().t()
    assert _rel(c, ref) < 1e-2, _rel(c, ref)
    assert torch.equal(c, ext().gemm_dense(a, b, pair=True))  # deterministic


def _moe_ref(x, top_idx, gate, w1, w2, w3, shared, act):
    T, d = x.shape
    E = w1.shape[0]
    k = top_idx.shape[1]
    eidx = top_idx.t().reshape(-1)
    perm = torch.argsort(eidx, stable=True)
    sizes = torch.bincount(eidx, minlength=E).tolist()
    rows = perm % T
    y = R.grouped_ffn(x[rows], sizes, w1, w2, w3, act)
    wgt = gate.t().reshape(-1)[perm]
    out = torch.zeros(T, d, device=x.device, dtype=torch.float32)
    out.index_add_(0, rows, y.float() * wgt[:, None])
    if shared is not None:
        out = out + shared.float()
    return R.sanitize(out, 1e3)


@pytest.mark.parametrize("act", ["swiglu", "gelu"])
@pytest.mark.parametrize("T,d,F,E,k", [(256, 256, 256, 4, 2), (1000, 512, 256, 8, 2), (512, 256, 512, 5, 3),
                                         (700, 256, 256, 64, 6)])
def test_moe_forward_backward(act, T, d, F, E, k):
    ext().gemm_error_reset()
    torch.manual_seed(1)
    x = (torch.randn(T, d, device=dev) * 0.5).to(torch.bfloat16)
    logits = torch.randn(T, E, device=dev)
    top_idx = torch.topk(logits, k, -1).indices
    gate = torch.softmax(logits.gather(1, top_idx), -1)
    w1 = (torch.randn(E, d, F, device=dev) * d ** -0.5).to(torch.bfloat16)
    w2 = (torch.randn(E, F, d, device=dev) * F ** -0.5).to(torch.bfloat16)
    w3 = (torch.randn(E, d, F, device=dev) * d ** -0.5).to(torch.bfloat16) if act == "swiglu" else None
    shared = (torch.randn(T, d, device=dev) * 0.1).to(torch.bfloat16)
    ins = [x, gate, w1, w2] + ([w3] if w3 is not None else [])
    xa = [t.clone().requires_grad_(True) for t in ins]
    out = KN.moe_forward(xa[0], top_idx, xa[1], xa[2], xa[3], xa[4] if w3 is not None else None, shared, act)
    xr = [t.detach().float().clone().requires_grad_(True) for t in ins]
    ref = _moe_ref(xr[0], top_idx, xr[1], xr[2], xr[3], xr[4] if w3 is not None else None, shared, act)
    assert _rel(out, ref) < 2e-2, _rel(out, ref)
    dout = torch.randn_like(ref)
    (out.float() * dout).sum().backward()
    (ref * dout).sum().backward()
    torch.cuda.synchronize()
    assert KN.gemm_error() == 0
    for name, a, r in zip(["x", "gate", "w1", "w2", "w3"], xa, xr):
        assert a.grad is not None, name
        err = _rel(a.grad, r.grad)
        assert err < 3e-2, (name, err)


def test_moe_weight_gradients_into_bf16_accumulators():
    """Expert weight gradients added into bf16 accumulators (a store with 16-bit gradients):
    the GEMM epilogue sums in fp32 and rounds once per add, so two backward passes match the
    fp32 accumulators to bf16 precision."""
    ext().gemm_error_reset()
    torch.manual_seed(3)
    T, d, F, E, k = 1024, 512, 256, 8, 2
    x = (torch.randn(T, d, device=dev) * 0.5).to(torch.bfloat16)
    logits = torch.randn(T, E, device=dev)
    top_idx = torch.topk(logits, k, -1).indices
    gate = torch.softmax(logits.gather(1, top_idx), -1)
    ws = [(torch.randn(E, d, F, device=dev) * d ** -0.5).to(torch.bfloat16),
          (torch.randn(E, F, d, device=dev) * F ** -0.5).to(torch.bfloat16),
          (torch.randn(E, d, F, device=dev) * d ** -0.5).to(torch.bfloat16)]
    dout = torch.randn(T, d, device=dev).to(torch.bfloat16)
    accs = {}
    for dt in (torch.float32, torch.bfloat16):
        wa = [w.clone().requires_grad_(True) for w in ws]
        for w in wa:
            w._ahb_grad_acc = torch.zeros(w.shape, dtype=dt, device=dev)
        for _ in range(2):
            out = KN.moe_forward(x, top_idx, gate, wa[0], wa[1], wa[2], None, "swiglu")
            out.backward(dout)
        torch.cuda.synchronize()
        accs[dt] = [w._ahb_grad_acc.float() for w in wa]
    assert KN.gemm_error() == 0
    for a, r in zip(accs[torch.bfloat16], accs[torch.float32]):
        assert _rel(a, r) < 1e-2, _rel(a, r)
