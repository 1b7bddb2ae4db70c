"""Causal flash attention kernel against the fp32 PyTorch reference."""
import pytest
import torch

from atomic_ai_hybrid_b200.ops import kernels as K
from atomic_ai_hybrid_b200.ops import reference as R

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("B,H,L,D", [(1, 2, 64, 64), (2, 3, 200, 128), (1, 2, 130, 96), (1, 1, 512, 128)])
def test_attention_fwd_bwd(B, H, L, D):
    torch.manual_seed(0)
    q, k, v = (torch.randn(B, H, L, D, device="cuda") for _ in range(3))
    scale = D ** -0.5
    qr, kr, vr = (t.clone().requires_grad_(True) for t in (q, k, v))
    ref = R.causal_attention(qr, kr, vr, scale)
    do = torch.randn_like(ref)
    ref.backward(do)
    qk, kk, vk = (t.to(torch.bfloat16).requires_grad_(True) for t in (q, k, v))
    out = K.attention(qk, kk, vk, scale)
    out.backward(do.to(torch.bfloat16))
    torch.testing.assert_close(out.float(), ref.detach(), atol=2e-2, rtol=2e-2)
    for a, b, n in ((qk.grad, qr.grad, "dq"), (kk.grad, kr.grad, "dk"), (vk.grad, vr.grad, "dv")):
        err = (a.float() - b).abs().max() / (b.abs().max() + 1e-6)
        assert err < 3e-2, (n, float(err))


@pytest.mark.parametrize("n", [2, 3, 7])
def test_source_mix(n):
    """BlockDAR source softmax kernel vs the PyTorch expression."""
    torch.manual_seed(n)
    T, dl, d = 300, 384, 768
    q = torch.randn(T, dl, device="cuda")
    ks = [torch.randn(T, dl, device="cuda") for _ in range(n)]
    ss = [torch.randn(T, d, device="cuda") for _ in range(n)]
    scale = dl ** -0.5
    qr, ksr, ssr = q.clone().requires_grad_(True), [k.clone().requires_grad_(True) for k in ks], \
        [s.clone().requires_grad_(True) for s in ss]
    w = torch.softmax(torch.stack([(qr * k).sum(-1) for k in ksr], 0) * scale, 0)
    ref = sum(w[i][:, None] * s for i, s in enumerate(ssr))
    g = torch.randn(T, d, device="cuda")
    ref.backward(g)
    qb = q.to(torch.bfloat16).requires_grad_(True)
    kb = [k.to(torch.bfloat16).requires_grad_(True) for k in ks]
    sb = [s.to(torch.bfloat16).requires_grad_(True) for s in ss]
    out = K.source_mix(qb, kb, sb, scale)
    out.backward(g.to(torch.bfloat16))
    torch.testing.assert_close(out.float(), ref.detach(), atol=3e-2, rtol=2e-2)
    for a, b in [(qb.grad, qr.grad)] + list(zip([k.grad for k in kb], [k.grad for k in ksr])) + \
            list(zip([s.grad for s in sb], [s.grad for s in ssr])):
        err = (a.float() - b).abs().max() / (b.abs().max() + 1e-6)
        assert err < 3e-2, float(err)
