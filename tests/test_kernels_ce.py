"""Fused LM-head cross entropy against the chunked PyTorch reference."""
import pytest
import torch

from atomic_ai_hybrid_b200.ops import kernels as KN
from atomic_ai_hybrid_b200.ops import reference as R

pytestmark = pytest.mark.gpu
dev = "cuda"


@pytest.mark.parametrize("T,d,V,ls", [(256, 256, 512, 0.0), (300, 512, 1024, 0.05), (1000, 256, 50304, 0.05)])
def test_fused_ce(T, d, V, ls):
    torch.manual_seed(0)
    h = (torch.randn(T, d, device=dev) * 0.5).to(torch.bfloat16).requires_grad_(True)
    W = (torch.randn(V, d, device=dev) * 0.05).requires_grad_(True)
    labels = torch.randint(0, V, (T,), device=dev)
    labels[::7] = -100
    s, c = KN.cross_entropy(h, labels, W, ls)
    (s / c).backward()
    h2 = h.detach().float().requires_grad_(True)
    W2 = W.detach().clone().requires_grad_(True)
    logits = (h2.to(torch.bfloat16) @ W2.to(torch.bfloat16).t()).float()
    s2, c2 = R.label_smoothed_ce(logits, labels, ls)
    (s2 / c2).backward()
    assert c.item() == c2.item()
    torch.testing.assert_close(s.float(), s2, rtol=2e-3, atol=1e-2)
    rel = lambda a, b: ((a.float() - b.float()).norm() / b.float().norm()).item()
    assert rel(h.grad, h2.grad) < 2e-2, rel(h.grad, h2.grad)
    assert rel(W.grad, W2.grad) < 2e-2, rel(W.grad, W2.grad)


@pytest.mark.parametrize("T,d,V,ls,chunk", [(1000, 256, 50304, 0.05, 256), (4096, 2048, 50304, 0.1, 8192)])
def test_fused_ce_chunks_and_production_head(T, d, V, ls, chunk, monkeypatch):
    """Backward in several row chunks (the last one partial) and the production head
    (d 2048, V 50304) against the fp32 reference on the same bf16 logits."""
    monkeypatch.setattr(KN, "CE_CHUNK_ROWS", chunk)
    torch.manual_seed(1)
    h = (torch.randn(T, d, device=dev) * 0.5).to(torch.bfloat16).requires_grad_(True)
    W = (torch.randn(V, d, device=dev) * 0.02).requires_grad_(True)
    labels = torch.randint(0, V, (T,), device=dev)
    labels[::5] = -100
    s, c = KN.cross_entropy(h, labels, W, ls)
    (s / c).backward()
    h2 = h.detach().float().requires_grad_(True)
    W2 = W.detach().clone().requires_grad_(True)
    logits = (h2.to(torch.bfloat16) @ W2.to(torch.bfloat16).t()).float()
    s2, c2 = R.label_smoothed_ce(logits, labels, ls)
    (s2 / c2).backward()
    assert c.item() == c2.item()
    torch.testing.assert_close(s.float(), s2, rtol=2e-3, atol=1e-2)
    rel = lambda a, b: ((a.float() - b.float()).norm() / b.float().norm()).item()
    assert rel(h.grad, h2.grad) < 2e-2, rel(h.grad, h2.grad)
    assert rel(W.grad, W2.grad) < 2e-2, rel(W.grad, W2.grad)


def test_fused_ce_forward_stores_no_logits():
    """The forward's peak memory stays far below one (T, V) bf16 logits tensor."""
    T, d, V = 4096, 512, 50304
    h = (torch.randn(T, d, device=dev) * 0.5).to(torch.bfloat16)
    W = (torch.randn(V, d, device=dev) * 0.02).to(torch.bfloat16)
    labels = torch.randint(0, V, (T,), device=dev)
    torch.cuda.synchronize()
    base = torch.cuda.memory_allocated()
    torch.cuda.reset_peak_memory_stats()
    with torch.no_grad():
        s, c = KN.cross_entropy(h, labels, W, 0.0)
    torch.cuda.synchronize()
    assert torch.isfinite(s) and c.item() == T
    assert torch.cuda.max_memory_allocated() - base < T * V * 2 // 4
