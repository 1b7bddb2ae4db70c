"""Context-parallel scan composition on the sm_100a kernels, one GPU: the sequence is cut into
segments, each segment's ``CPGroup`` composes its output from the other segments' final
states and transfers (the all-gather replaced by the segments' own results, computed from the
same inputs so the gradients cross segments as through the collective), and the outputs and
input gradients match the unsplit kernel scan."""
import math

import pytest
import torch
import torch.nn.functional as F

from atomic_ai_hybrid_b200 import ops
from atomic_ai_hybrid_b200.parallel.cp import CPGroup

pytestmark = pytest.mark.gpu
dev = "cuda"


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


class _LocalCP(CPGroup):
    """Rank ``rank`` of ``world`` segments whose gathers return the given per-segment lists
    (transfers first, then final states: the order in which the scans gather them)."""

    def __init__(self, world, rank, lists):
        super().__init__(world, rank)
        self._lists = list(lists)

    def gather(self, t):
        return self._lists.pop(0)


def _run_segments(scan, ins, W, finals):
    outs = []
    for r in range(W):
        seg = [t.chunk(W, 1)[r] if t.dim() > 1 else t for t in ins]
        outs.append(scan(_LocalCP(W, r, finals), seg))
    return torch.cat(outs, 1)


def test_cp_gdn_on_kernels_matches_unsplit():
    ops.set_impl("cuda")
    B, L, H, D, W = 1, 512, 2, 128, 2
    g_ = torch.Generator(device=dev).manual_seed(0)
    bf = torch.bfloat16
    q = F.normalize(torch.randn(B, L, H, D, generator=g_, device=dev), dim=-1).to(bf)
    k = F.normalize(torch.randn(B, L, H, D, generator=g_, device=dev), dim=-1).to(bf)
    v = torch.randn(B, L, H, D, generator=g_, device=dev).to(bf)
    g = -F.softplus(torch.randn(B, L, H, D, generator=g_, device=dev))
    b = torch.sigmoid(torch.randn(B, L, H, D, generator=g_, device=dev)).to(bf)
    w = torch.sigmoid(torch.randn(B, L, H, D, generator=g_, device=dev)).to(bf)
    do = torch.randn(B, L, H, D, generator=g_, device=dev).to(bf)
    base = [q, k, v, g, b, w]

    full = [t.clone().requires_grad_(True) for t in base]
    o_full = ops.gdn2(full[0], full[1], full[2], full[5], full[4], full[3], 1.0, 64)
    (o_full.float() * do.float()).sum().backward()

    xs = [t.clone().requires_grad_(True) for t in base]
    Ts, Ss = [], []
    eye = torch.eye(D, device=dev).expand(B, H, D, D).contiguous()
    for r in range(W):
        sq, sk, sv, sg, sb, sw = (t.chunk(W, 1)[r] for t in xs)
        _, S = ops.gdn2(sq, sk, sv, sw, sb, sg, 1.0, 64, return_final=True)
        _, T = ops.gdn2(sq, sk, torch.zeros_like(sv), sw, sb, sg, 1.0, 64, h0=eye, return_final=True)
        Ts.append(T)
        Ss.append(S)
    o_cp = _run_segments(lambda cp, s: cp.gdn2_scan(s[0], s[1], s[2], s[3], s[4], s[5], 1.0, 64), xs, W,
                         [Ts, Ss] * 1)
    assert _rel(o_cp, o_full) < 2e-2, _rel(o_cp, o_full)
    (o_cp.float() * do.float()).sum().backward()
    for name, a, r in zip("qkvgbw", xs, full):
        assert _rel(a.grad, r.grad) < 3e-2, (name, _rel(a.grad, r.grad))


def test_cp_ssd_on_kernels_matches_unsplit():
    ops.set_impl("cuda")
    B, L, H, P, N, W = 1, 512, 3, 64, 128, 2
    g_ = torch.Generator(device=dev).manual_seed(1)
    bf = torch.bfloat16
    x = torch.randn(B, L, H, P, generator=g_, device=dev).to(bf)
    dt = F.softplus(torch.randn(B, L, H, P, generator=g_, device=dev) - 1.0).clamp(1e-2, 1.0).to(bf)
    A = -torch.exp(torch.rand(H, generator=g_, device=dev) * math.log(16.0))
    Bm = (torch.randn(B, L, N, generator=g_, device=dev) / math.sqrt(N)).to(bf)
    Cm = (torch.randn(B, L, N, generator=g_, device=dev) / math.sqrt(N)).to(bf)
    dy = torch.randn(B, L, H, P, generator=g_, device=dev).to(bf)
    base = [dt, A, Bm, Cm, x]

    full = [t.clone().requires_grad_(True) for t in base]
    y_full = ops.ssd(*full, 64)
    (y_full.float() * dy.float()).sum().backward()

    xs = [t.clone().requires_grad_(True) for t in base]
    Ts, Ss = [], []
    for r in range(W):
        sdt, sB, sC, sx = (t.chunk(W, 1)[r] for t in (xs[0], xs[2], xs[3], xs[4]))
        _, S = ops.ssd(sdt, xs[1], sB, sC, sx, 64, return_final=True)
        _, T = ops.ssd(sdt, xs[1], sB, sC, torch.zeros_like(sx), 64, state0=torch.ones_like(S), return_final=True)
        Ts.append(T)
        Ss.append(S)
    y_cp = _run_segments(lambda cp, s: cp.ssd_scan(s[0], s[1], s[2], s[3], s[4], 64), xs, W, [Ts, Ss])
    assert _rel(y_cp, y_full) < 2e-2, _rel(y_cp, y_full)
    (y_cp.float() * dy.float()).sum().backward()
    for name, a, r in zip(["dt", "A", "B", "C", "x"], xs, full):
        assert _rel(a.grad, r.grad) < 5e-2, (name, _rel(a.grad, r.grad))
