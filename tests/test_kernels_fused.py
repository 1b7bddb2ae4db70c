"""Fused layer-glue kernels (fused_norm.cu) against plain PyTorch fp32 references."""
import math

import pytest
import torch
import torch.nn.functional as F

from atomic_ai_hybrid_b200.ops import kernels as K
from atomic_ai_hybrid_b200.ops import reference as R

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _close(a, b, rtol, atol, name=""):
    torch.testing.assert_close(a.float(), b.float(), rtol=rtol, atol=atol, msg=name)


def _rms(x, scale, eps=1e-6):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * scale


@pytest.mark.parametrize("sdg", [True, False])
def test_add_rmsnorm(sdg):
    torch.manual_seed(0)
    M, D, clip = 300, 2048, 5e2
    x = (torch.randn(M, D, device=DEV) * 3).to(torch.bfloat16)
    delta = (torch.randn(M, D, device=DEV) * 3).to(torch.bfloat16)
    x[0, :5] = 400
    delta[0, :5] = 200  # clipped entries
    scale = torch.rand(D, device=DEV) + 0.5
    xr, dr, sr = (t.float().clone().requires_grad_(True) for t in (x, delta, scale))
    s = (x.float() + delta.float()).to(torch.bfloat16).float()
    mask = (s.abs() < clip).float()
    xo_ref = s.clamp(-clip, clip)
    # reference graph: the clip gradient is the mask of the rounded sum
    xo_g = (xr + dr) * mask + (xo_ref - (xr + dr) * mask).detach()
    y_ref = _rms(xo_g, sr)
    gy = torch.randn(M, D, device=DEV).to(torch.bfloat16)
    gres = torch.randn(M, D, device=DEV).to(torch.bfloat16)
    (y_ref * gy.float()).sum().add_((xo_g * gres.float()).sum()).backward()

    xk, dk = x.clone().requires_grad_(True), delta.clone().requires_grad_(True)
    sk = scale.clone().requires_grad_(True)
    xo, y = K.add_rmsnorm(xk, dk, sk, clip, 1e-6, sanitize_delta_grad=sdg)
    torch.autograd.backward([y, xo], [gy, gres])
    _close(xo, xo_ref, 0, 0, "xo")
    _close(y, y_ref.detach(), 1e-2, 1e-2, "y")
    _close(xk.grad, xr.grad, 2e-2, 2e-2, "dx")
    dref = xr.grad.clamp(-1e3, 1e3) if sdg else xr.grad
    _close(dk.grad, dref, 2e-2, 2e-2, "ddelta")
    _close(sk.grad, sr.grad, 1e-3, 1e-2, "dscale")


@pytest.mark.parametrize("zclip,oclip", [(1e2, math.inf), (math.inf, 3e2)])
def test_norm_gate(zclip, oclip):
    torch.manual_seed(1)
    M, D = 257, 2048
    x = (torch.randn(M, D, device=DEV) * 2).to(torch.bfloat16)
    zfull = (torch.randn(M, 2 * D, device=DEV) * 4).to(torch.bfloat16)
    z = zfull[:, D:]  # strided rows, as Mamba2's `res`
    z[0, :4] = 150
    scale = torch.rand(D, device=DEV) * 200 + 0.5
    xr, zr, sr = (t.float().clone().requires_grad_(True) for t in (x, z, scale))
    y_ref = (_rms(xr, sr) * F.silu(zr.clamp(-zclip, zclip))).clamp(-oclip, oclip)
    gy = torch.randn(M, D, device=DEV).to(torch.bfloat16)
    (y_ref * gy.float()).sum().backward()
    xk, zk, sk = x.clone().requires_grad_(True), zfull.clone().requires_grad_(True), scale.clone().requires_grad_(True)
    y = K.norm_gate(xk, zk[:, D:], sk, 1e-6, zclip, oclip)
    y.backward(gy)
    _close(y, y_ref.detach(), 1e-2, 5e-2, "y")
    _close(xk.grad, xr.grad, 2e-2, 5e-2, "dx")
    _close(zk.grad[:, D:], zr.grad, 2e-2, 5e-2, "dz")
    assert not zk.grad[:, :D].any()
    _close(sk.grad, sr.grad, 1e-3, 2e-2, "dscale")


def test_gdn_gates():
    torch.manual_seed(2)
    B, L, H, Dh = 2, 64, 4, 128
    d = H * Dh
    bp, wp, fp = ((torch.randn(B, L, d, device=DEV) * 3).to(torch.bfloat16) for _ in range(3))
    fp[0, 0, 2 * Dh:2 * Dh + 3] = float("inf")  # in head 2, whose decay_a is clamped
    a = torch.tensor([0.5, -1.0, 25.0, 2.0], device=DEV)
    br, wr, fr, ar = (t.float().clone().requires_grad_(True) for t in (bp, wp, fp, a))
    bg_ref, wg_ref = torch.sigmoid(br), torch.sigmoid(wr)
    g = -torch.exp(ar.clamp(-20, 20)).repeat_interleave(Dh)[None, None] * F.softplus(fr)
    g_ref = torch.nan_to_num(g, nan=0.0, posinf=0.0, neginf=-20.0).clamp(-1e3, 1e3)
    dbg, dwg = (torch.randn(B, L, d, device=DEV).to(torch.bfloat16) for _ in range(2))
    dg = torch.randn(B, L, d, device=DEV)
    ((bg_ref * dbg.float()).sum() + (wg_ref * dwg.float()).sum() + (g_ref * dg).sum()).backward()
    bk, wk, fk, ak = (t.clone().requires_grad_(True) for t in (bp, wp, fp, a))
    bg, wg, gk = K.gdn_gates(bk, wk, fk, ak, Dh)
    torch.autograd.backward([bg, wg, gk], [dbg, dwg, dg])
    _close(bg, bg_ref.detach(), 1e-2, 1e-2, "b")
    _close(wg, wg_ref.detach(), 1e-2, 1e-2, "w")
    _close(gk, g_ref.detach(), 1e-4, 1e-4, "g")
    _close(bk.grad, br.grad, 2e-2, 1e-2, "dbp")
    _close(wk.grad, wr.grad, 2e-2, 1e-2, "dwp")
    _close(fk.grad, fr.grad, 2e-2, 1e-2, "dfp")
    assert torch.isfinite(ak.grad).all()
    _close(ak.grad[[0, 1, 3]], ar.grad[[0, 1, 3]], 1e-3, 1e-2, "da")
    assert float(ak.grad[2]) == 0.0


def test_l2norm_heads():
    torch.manual_seed(3)
    x = (torch.randn(3, 50, 4, 128, device=DEV) * 2).to(torch.bfloat16)
    xr = x.float().clone().requires_grad_(True)
    y_ref = R.safe_l2norm(xr, 1e-12)
    dy = torch.randn_like(xr) * 600  # partly beyond the sanitizer's +-1e3
    (y_ref * dy.clamp(-1e3, 1e3)).sum().backward()
    xk = x.clone().requires_grad_(True)
    y = K.l2norm_heads(xk)
    y.backward(dy.to(torch.bfloat16))
    _close(y, y_ref.detach(), 1e-2, 1e-2, "y")
    _close(xk.grad, xr.grad, 2e-2, 2e-1, "dx")


def test_dt_act():
    torch.manual_seed(4)
    u = (torch.randn(4, 64, 256, device=DEV) * 3 - 3).to(torch.bfloat16)
    ur = u.clone().requires_grad_(True)
    ref = F.softplus(ur).clamp(1e-2, 1.0)
    g = torch.randn_like(ref)
    ref.backward(g)
    uk = u.clone().requires_grad_(True)
    dt = K.dt_act(uk)
    dt.backward(g)
    _close(dt, ref.detach(), 0, 0, "dt")
    _close(uk.grad, ur.grad, 2e-2, 1e-2, "du")


def test_fused_model_matches_unfused():
    """The interleaved stack with fused residual/norm glue equals the unfused path."""
    from atomic_ai_hybrid_b200 import get_preset, ops
    from atomic_ai_hybrid_b200.models import HybridMoEModel
    from atomic_ai_hybrid_b200.training.loss import compute_loss
    ops.set_impl("cuda")
    cfg = get_preset("hybrid_1b", d_model=256, n_heads=2, n_heads_ssm=4, num_layers=2, d_ff=256,
                     n_routed_experts=8, top_k=2, vocab_size=1024, d_state=128, router_noise_std=0.0)
    torch.manual_seed(0)
    m = HybridMoEModel(cfg, compute_dtype=torch.bfloat16).to(DEV)
    for p in m.parameters():
        if p.ndim >= 2:
            p.data = p.data.to(torch.bfloat16)
    ids = torch.randint(0, cfg.vocab_size, (2, 129), device=DEV)
    batch = {"input_ids": ids[:, :-1], "labels": ids[:, 1:]}
    out = {}
    for fused in (True, False):
        m.zero_grad(set_to_none=True)
        m._fused_residuals = (lambda x, f=fused: f and x.is_cuda)
        loss, _ = compute_loss(m, batch, deterministic=True)
        loss.backward()
        out[fused] = (loss.detach(), {n: p.grad.float().clone() for n, p in m.named_parameters()
                                      if p.grad is not None})
    del m._fused_residuals
    _close(out[True][0], out[False][0], 2e-3, 2e-3, "loss")
    for n, g in out[False][1].items():
        gf = out[True][1][n]
        rel = (gf - g).norm() / (g.norm() + 1e-12)
        assert rel < 5e-2, (n, float(rel))


@pytest.mark.parametrize("op", ["gdn", "ssd"])
def test_saved_scan_intermediates_match_recompute(op, monkeypatch):
    """The backward on the forward's saved chunk intermediates equals the recomputing one."""
    torch.manual_seed(5)
    B, L = 2, 256
    if op == "gdn":
        H, D = 2, 128
        q = F.normalize(torch.randn(B, L, H, D, device=DEV), dim=-1).to(torch.bfloat16)
        k = F.normalize(torch.randn(B, L, H, D, device=DEV), dim=-1).to(torch.bfloat16)
        v = torch.randn(B, L, H, D, device=DEV).to(torch.bfloat16)
        b = torch.sigmoid(torch.randn(B, L, H, D, device=DEV)).to(torch.bfloat16)
        w = torch.sigmoid(torch.randn(B, L, H, D, device=DEV)).to(torch.bfloat16)
        g = -F.softplus(torch.randn(B, L, H, D, device=DEV))
        inputs = [q, k, v, w, b, g]
        run = lambda t: K.gdn2(*t, 1.0, 64)  # noqa: E731
    else:
        H, P, N = 4, 64, 128
        dt = F.softplus(torch.randn(B, L, H, P, device=DEV) - 3).to(torch.bfloat16)
        A = -torch.exp(torch.rand(H, device=DEV) * 2)
        Bm = torch.randn(B, L, N, device=DEV).to(torch.bfloat16)
        Cm = torch.randn(B, L, N, device=DEV).to(torch.bfloat16)
        x = torch.randn(B, L, H, P, device=DEV).to(torch.bfloat16)
        inputs = [dt, A, Bm, Cm, x]
        run = lambda t: K.ssd(*t, 64)  # noqa: E731
    grads = {}
    for recompute in (False, True):
        monkeypatch.setattr(K, "SCAN_RECOMPUTE", recompute)
        ts = [t.clone().requires_grad_(True) for t in inputs]
        out = run(ts)
        out.backward(torch.ones_like(out))
        grads[recompute] = [t.grad.float() for t in ts]
    for a, r in zip(grads[False], grads[True]):  # equal up to atomics' summation order
        torch.testing.assert_close(a, r, rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("E,k,d", [(32, 4, 2048), (8, 2, 256), (64, 6, 512)])
def test_fused_router_matches_torch(E, k, d, monkeypatch):
    """Fused router kernel vs the PyTorch router: selection, gates, statistics, gradients."""
    from atomic_ai_hybrid_b200 import get_preset, ops
    from atomic_ai_hybrid_b200.models.moe import MoE
    ops.set_impl("cuda")
    cfg = get_preset("hybrid_1b", d_model=d, n_routed_experts=E, top_k=k, router_noise_std=0.0)
    torch.manual_seed(6)
    moe = MoE(cfg).to(DEV)
    moe.expert_bias.data = torch.randn(E, device=DEV) * 0.05
    x = (torch.randn(700, d, device=DEV) * 2).to(torch.bfloat16)
    res = {}
    for fused in (True, False):
        monkeypatch.setattr(K, "router_supported", lambda *a, f=fused: f)
        moe.zero_grad(set_to_none=True)
        xx = x.clone().requires_grad_(True)
        st = {}
        top, gate = moe.route(xx, st)
        wg = torch.linspace(0.5, 1.5, gate.numel(), device=DEV).view_as(gate)
        loss = (gate * wg).sum() + 3.0 * st["aux_loss"] + 0.5 * st["z_loss"] + st["router_collinearity"]
        loss.backward()
        res[fused] = (top, gate.detach(), {kk: v.detach().float() for kk, v in st.items()}, xx.grad.float(),
                      moe.router.grad.clone(), moe.router_temp.grad.clone())
    (t1, g1, s1, dx1, dr1, dt1), (t0, g0, s0, dx0, dr0, dt0) = res[True], res[False]
    assert torch.equal(t1, t0)
    _close(g1, g0, 1e-4, 1e-5, "gate")
    for kk in ("aux_loss", "z_loss", "norm_x_mean", "norm_x_max", "norm_x_min", "max_abs_logit_preclip",
               "assignment_frac", "expert_utilization"):
        _close(s1[kk], s0[kk], 1e-4, 1e-4, kk)
    _close(dx1, dx0, 2e-2, 1e-4, "dx")
    _close(dr1, dr0, 1e-3, 1e-5, "drouter")
    _close(dt1, dt0, 1e-3, 1e-6, "dtemp")


def test_linear_multi_grads():
    """Several projections of one input: outputs, input gradient and weight gradients
    (added straight into fp32 accumulators) equal the plain PyTorch expressions."""
    torch.manual_seed(8)
    x = torch.randn(3, 100, 256, device=DEV).to(torch.bfloat16)
    ws = [(torch.randn(256, n, device=DEV) * 0.05).to(torch.bfloat16) for n in (256, 128, 512)]
    bs = [None, torch.randn(128, device=DEV), torch.randn(512, device=DEV)]
    accs = [torch.zeros(w.shape, device=DEV) for w in ws]
    wk = [w.clone().requires_grad_(True) for w in ws]
    for w, a in zip(wk, accs):
        w._ahb_grad_acc = a
    bk = [None if b is None else b.clone().requires_grad_(True) for b in bs]
    xk = x.clone().requires_grad_(True)
    outs = K.linear_multi(xk, list(zip(wk, bk)))
    gs = [torch.randn_like(o) for o in outs]
    torch.autograd.backward(list(outs), gs)
    xr = x.float().clone().requires_grad_(True)
    wr = [w.float().clone().requires_grad_(True) for w in ws]
    br = [None if b is None else b.clone().requires_grad_(True) for b in bs]
    refs = [xr @ w + (0 if b is None else b) for w, b in zip(wr, br)]
    torch.autograd.backward(refs, [g.float() for g in gs])
    for o, r in zip(outs, refs):
        _close(o, r.detach(), 2e-2, 5e-2, "y")
    _close(xk.grad, xr.grad, 2e-2, 1e-1, "dx")
    for a, w, wkk in zip(accs, wr, wk):
        assert wkk.grad is None  # accumulated into the fp32 buffer instead
        _close(a, w.grad, 1e-2, 1e-1, "dW")
    for b, r in zip(bk, br):
        if b is not None:
            _close(b.grad, r.grad, 1e-3, 1e-2, "db")


@pytest.mark.parametrize("M,N", [(16384, 2048), (1000, 136), (7, 1024)])
def test_bias_grad_acc_matches_column_sums(M, N):
    from atomic_ai_hybrid_b200.ops._ext import ext
    dev = torch.device("cuda", 0)
    dy = torch.randn(M, N, device=dev).to(torch.bfloat16)
    acc = torch.randn(N, device=dev)
    ref = acc + dy.float().sum(0)
    ext().bias_grad_acc(dy, acc)
    torch.testing.assert_close(acc, ref, rtol=1e-4, atol=1e-3)


@pytest.mark.parametrize("gated,zclip,oclip", [(True, 1e2, math.inf), (True, math.inf, 3e2), (False, math.inf, math.inf)])
def test_tp_norm_matches_full_width(gated, zclip, oclip, monkeypatch):
    """Head-split norm kernels (ops.kernels.tp_norm) on one GPU: two ranks holding the same
    piece are emulated by an all-reduce that doubles the row sums, so each rank's output and
    gradients equal the first half of a full-width (2 D) norm of the piece repeated twice."""
    import torch.distributed as dist
    monkeypatch.setattr(dist, "all_reduce", lambda t, group=None: t.mul_(2))
    tp = type("G", (), {"group": None})()
    torch.manual_seed(2)
    M, D = 129, 1024
    x = (torch.randn(M, D, device=DEV) * 2).to(torch.bfloat16)
    zfull = (torch.randn(M, 2 * D, device=DEV) * 4).to(torch.bfloat16)
    z = zfull[:, D:]  # strided rows, as Mamba2's `res`
    z[0, :4] = 150
    scale = torch.rand(D, device=DEV) * 2 + 0.5
    gy = torch.randn(M, D, device=DEV).to(torch.bfloat16)
    xr, zr, sr = (torch.cat([t, t], -1).float().clone().requires_grad_(True) for t in (x, z, scale))
    y_ref = _rms(xr, sr)
    if gated:
        y_ref = y_ref * F.silu(zr.clamp(-zclip, zclip))
    y_ref = y_ref.clamp(-oclip, oclip)
    (y_ref * torch.cat([gy, gy], -1).float()).sum().backward()
    xk, zk, sk = x.clone().requires_grad_(True), zfull.clone().requires_grad_(True), scale.clone().requires_grad_(True)
    y = K.tp_norm(xk, zk[:, D:] if gated else None, sk, 1e-6, 2 * D, tp, zclip, oclip)
    y.backward(gy)
    _close(y, y_ref[:, :D].detach(), 1e-2, 5e-2, "y")
    _close(xk.grad, xr.grad[:, :D], 2e-2, 5e-2, "dx")
    if gated:
        _close(zk.grad[:, D:], zr.grad[:, :D], 2e-2, 5e-2, "dz")
        assert not zk.grad[:, :D].any()
    _close(sk.grad, sr.grad[:D], 1e-3, 2e-2, "dscale")


def test_shared_expert_swiglu():
    """silu(a) * b kernels (shared expert of the SwiGLU configurations) against fp32 autograd."""
    torch.manual_seed(3)
    a = (torch.randn(1000, 264, device=DEV) * 3).to(torch.bfloat16)
    b = torch.randn(1000, 264, device=DEV).to(torch.bfloat16)
    dh = torch.randn(1000, 264, device=DEV).to(torch.bfloat16)
    ar, br = a.float().requires_grad_(True), b.float().requires_grad_(True)
    (F.silu(ar) * br).backward(dh.float())
    ak, bk = a.clone().requires_grad_(True), b.clone().requires_grad_(True)
    h = K.swiglu(ak, bk)
    h.backward(dh)
    _close(h, F.silu(a.float()) * b.float(), 1e-2, 1e-2, "h")
    _close(ak.grad, ar.grad, 1e-2, 1e-2, "da")
    _close(bk.grad, br.grad, 1e-2, 1e-2, "db")
