"""Plain-PyTorch restatements of the reference's numerical kernels.

These are the oracles every CUDA kernel of this package is tested against, and
they are also the op implementations of the unfused eager baseline model.  They
are written from the mathematics the reference states, in PyTorch:

* GDN-2 gated delta rule with per-channel decay/erase/write gates --
  token-serial ground truth (reference `atomic_ops/gdn2_wy_reference.py:33-56`)
  and the chunked WY form with the reference's clip/nan guards
  (`atomic_ops/gdn2_wy_reference.py:59-152`).
* Mamba2 SSD with per-channel ``dt`` and per-head ``A`` -- chunked form with the
  reference's clip discipline (`atomic_ops/mamba2_ssd_reference.py:56-179`) and a
  token-serial ground truth.

Shapes follow the reference: sequence tensors are ``(B, L, H, D)``.
All arithmetic is done in fp32 (or fp64 when the inputs are fp64).
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.nn.functional as F

Tensor = torch.Tensor


def sanitize(x: Tensor, clip: float) -> Tensor:
    """``nan_to_num(clip(x, -c, c))`` -- the reference's guard at kernel boundaries."""
    return torch.nan_to_num(x.clamp(-clip, clip), nan=0.0, posinf=clip, neginf=-clip)


def _nan_guard(x: Tensor, big: float = 1e4) -> Tensor:
    return torch.nan_to_num(x, nan=0.0, posinf=big, neginf=-big)


def _acc_dtype(t: Tensor) -> torch.dtype:
    return torch.float64 if t.dtype == torch.float64 else torch.float32


# --------------------------------------------------------------------------
# GDN-2
# --------------------------------------------------------------------------
def gdn2_token_serial(q, k, v, g, b, w, scale: float = 1.0, h0: Optional[Tensor] = None):
    """Token-serial GDN-2 recurrence (ground truth).

    For every token: ``h <- diag(e^g) h``; ``v' = w*v - (b*k)^T h``;
    ``h += k v'^T``; ``o = h^T (q*scale)``.  ``g`` is the per-channel log-decay.
    Returns ``(o, h_final)`` with ``o`` in the dtype of ``q`` and ``h`` fp32/fp64.
    """
    B, L, H, D = q.shape
    Dv = v.shape[-1]
    acc = _acc_dtype(q)
    h = torch.zeros(B, H, D, Dv, dtype=acc, device=q.device) if h0 is None else h0.to(acc).clone()
    alpha = torch.exp(g.to(acc))
    outs = []
    for t in range(L):
        h = h * alpha[:, t, :, :, None]
        bk = (b[:, t] * k[:, t]).to(acc)
        erase = torch.einsum("bhd,bhdv->bhv", bk, h)
        v_new = (w[:, t] * v[:, t]).to(acc) - erase
        h = h + torch.einsum("bhd,bhv->bhdv", k[:, t].to(acc), v_new)
        outs.append(torch.einsum("bhdv,bhd->bhv", h, (q[:, t] * scale).to(acc)))
    return torch.stack(outs, 1).to(q.dtype), h


def gdn2_chunk_prepare(q_c, k_c, v_c, g_c, b_c, w_c, scale: float):
    """Intra-chunk quantities of the WY form for one chunk ``(B, C, H, D)``.

    Returns ``Aqk (B,H,C,C)``, ``w_pseudo (B,C,H,D)``, ``u (B,C,H,Dv)``,
    ``kg``, ``qg`` ``(B,C,H,D)`` and ``gc_last (B,H,D)``.  ``A = (I+Akk)^-1`` is
    taken with a batched triangular solve (same matrix the reference builds with
    its row recursion, reference `atomic_ops/gdn2_wy_reference.py:18-30`).
    """
    acc = _acc_dtype(q_c)
    C = q_c.shape[1]
    gc = torch.cumsum(g_c.to(acc), dim=1)                     # (B,C,H,D)
    gcb = gc.permute(0, 2, 1, 3)                               # (B,H,C,D)
    ediff = torch.exp((gcb[:, :, :, None, :] - gcb[:, :, None, :, :]).clamp(-20.0, 20.0))
    qb = q_c.permute(0, 2, 1, 3).to(acc)
    kb = k_c.permute(0, 2, 1, 3).to(acc)
    bb = b_c.permute(0, 2, 1, 3).to(acc)
    causal = torch.tril(torch.ones(C, C, dtype=acc, device=q_c.device))
    strict = torch.tril(torch.ones(C, C, dtype=acc, device=q_c.device), -1)
    Aqk = scale * torch.einsum("bhid,bhijd,bhjd->bhij", qb, ediff, kb) * causal
    Akk = torch.einsum("bhid,bhijd,bhjd->bhij", bb * kb, ediff, kb) * strict
    Aqk = _nan_guard(Aqk)
    Akk = _nan_guard(Akk)
    eye = torch.eye(C, dtype=acc, device=q_c.device).expand_as(Akk)
    A = torch.linalg.solve_triangular(eye + Akk, eye, upper=False, unitriangular=True)
    A = _nan_guard(A)
    kb_dec = (b_c.to(acc) * k_c.to(acc)) * torch.exp(gc)
    w_pseudo = _nan_guard(torch.einsum("bhij,bjhd->bihd", A, kb_dec))
    u = _nan_guard(torch.einsum("bhij,bjhv->bihv", A, (w_c * v_c).to(acc)))
    gc_last = gc[:, -1]
    kg = k_c.to(acc) * torch.exp(gc_last[:, None] - gc)
    qg = q_c.to(acc) * torch.exp(gc)
    return Aqk, w_pseudo, u, kg, qg, gc_last


def gdn2_chunk_step(h, Aqk, w_pseudo, u, kg, qg, gc_last, scale: float):
    """Inter-chunk step of the WY form: returns ``(h_next, o_chunk, v_new)``."""
    v_new = u - torch.einsum("bihd,bhdv->bihv", w_pseudo, h)
    qh = torch.einsum("bihd,bhdv->bihv", qg, h)
    intra = torch.einsum("bhij,bjhv->bihv", Aqk, v_new)
    o = _nan_guard(scale * qh + intra)
    write = torch.einsum("bihd,bihv->bhdv", kg, v_new)
    h_new = h * torch.exp(gc_last)[..., None] + write
    h_new = sanitize(h_new, 1e4)
    return h_new, o, v_new


def gdn2_chunked(q, k, v, g, b, w, scale: float = 1.0, chunk_size: int = 64,
                 h0: Optional[Tensor] = None, checkpoint_chunks: bool = False):
    """Chunked WY GDN-2 (reference `gdn2_chunked_wy_reference`).  Differentiable."""
    B, L, H, D = q.shape
    Dv = v.shape[-1]
    assert L % chunk_size == 0, f"seq_len={L} must be divisible by chunk_size={chunk_size}"
    acc = _acc_dtype(q)
    h = torch.zeros(B, H, D, Dv, dtype=acc, device=q.device) if h0 is None else h0.to(acc)

    def one(h, qc, kc, vc, gcn, bc, wc):
        prep = gdn2_chunk_prepare(qc, kc, vc, gcn, bc, wc, scale)
        h2, o, _ = gdn2_chunk_step(h, *prep, scale)
        return h2, o

    outs = []
    for s in range(0, L, chunk_size):
        sl = slice(s, s + chunk_size)
        args = (h, q[:, sl], k[:, sl], v[:, sl], g[:, sl], b[:, sl], w[:, sl])
        if checkpoint_chunks and torch.is_grad_enabled():
            import torch.utils.checkpoint as ckpt
            h, o = ckpt.checkpoint(one, *args, use_reentrant=False)
        else:
            h, o = one(*args)
        outs.append(o)
    return torch.cat(outs, 1).to(q.dtype), h


# --------------------------------------------------------------------------
# Mamba2 SSD
# --------------------------------------------------------------------------
def ssd_token_serial(dt, A, Bm, Cm, x, state0: Optional[Tensor] = None):
    """Token-serial SSD: ``s_t = e^{dt_t A} s_{t-1} + (dt_t x_t) B_t^T``; ``y_t = s_t C_t``.

    ``dt, x: (B,L,H,P)``, ``A: (H,)``, ``B, C: (B,L,N)``.  State is ``(B,H,P,N)``.
    """
    Bsz, L, H, P = dt.shape
    N = Bm.shape[-1]
    acc = _acc_dtype(dt)
    s = torch.zeros(Bsz, H, P, N, dtype=acc, device=dt.device) if state0 is None else state0.to(acc).clone()
    Af = A.to(acc)
    ys = []
    for t in range(L):
        dA = (dt[:, t].to(acc) * Af[None, :, None]).clamp(-20.0, 20.0)
        s = s * torch.exp(dA)[..., None] + torch.einsum("bhp,bn->bhpn", dt[:, t].to(acc) * x[:, t].to(acc), Bm[:, t].to(acc))
        ys.append(torch.einsum("bhpn,bn->bhp", s, Cm[:, t].to(acc)))
    return torch.stack(ys, 1).to(x.dtype), s


def ssd_chunk(dt_c, A, B_c, C_c, x_c, state_prev):
    """One chunk of the reference SSD with its exact clip discipline
    (reference `atomic_ops/mamba2_ssd_reference.py:56-148`)."""
    acc = state_prev.dtype
    Cs = dt_c.shape[1]
    dA = sanitize(dt_c.to(acc) * A.to(acc)[None, None, :, None], 20.0)
    cum = sanitize(torch.cumsum(dA, dim=1), 1e4)                           # (b,C,h,p)
    diff = cum[:, :, None] - cum[:, None, :]                                 # (b,i,j,h,p)
    causal = torch.tril(torch.ones(Cs, Cs, dtype=acc, device=dt_c.device))[None, :, :, None, None]
    Lm = sanitize(torch.exp(diff.clamp(-20.0, 20.0)) * causal, 1e6)
    CB = sanitize(torch.einsum("bis,bjs->bij", C_c.to(acc), B_c.to(acc)), 1e4)
    dBx = sanitize(dt_c.to(acc) * x_c.to(acc), 1e4)
    y_diag = sanitize(torch.einsum("bijhp,bij,bjhp->bihp", Lm, CB, dBx), 1e4)
    dte = sanitize(torch.exp((cum[:, -1:] - cum).clamp(-20.0, 20.0)), 1e6)
    state_end = sanitize(torch.einsum("bcs,bchp->bhps", B_c.to(acc), dBx * dte), 1e4)
    decay_h = torch.exp(cum.clamp(-20.0, 0.0))
    y_off = sanitize(torch.einsum("bis,bhps->bihp", C_c.to(acc), state_prev) * decay_h, 1e4)
    dce = torch.exp(cum[:, -1].clamp(-20.0, 0.0))
    state_new = sanitize(state_prev * dce[..., None] + state_end, 1e4)
    return sanitize(y_diag + y_off, 1e4), state_new


def ssd_chunked(dt, A, Bm, Cm, x, chunk_size: int = 64, state0: Optional[Tensor] = None,
                checkpoint_chunks: bool = False):
    """Chunked SSD (reference `mamba2_ssd_reference`).  Differentiable."""
    Bsz, L, H, P = dt.shape
    N = Bm.shape[-1]
    assert L % chunk_size == 0
    acc = _acc_dtype(dt)
    s = torch.zeros(Bsz, H, P, N, dtype=acc, device=dt.device) if state0 is None else state0.to(acc)
    ys = []
    for st in range(0, L, chunk_size):
        sl = slice(st, st + chunk_size)
        args = (dt[:, sl], A, Bm[:, sl], Cm[:, sl], x[:, sl], s)
        if checkpoint_chunks and torch.is_grad_enabled():
            import torch.utils.checkpoint as ckpt
            y, s = ckpt.checkpoint(ssd_chunk, *args, use_reentrant=False)
        else:
            y, s = ssd_chunk(*args)
        ys.append(y)
    return torch.cat(ys, 1).to(x.dtype), s


# --------------------------------------------------------------------------
# Small ops
# --------------------------------------------------------------------------
def rmsnorm(x: Tensor, scale: Tensor, eps: float = 1e-6) -> Tensor:
    """Flax ``nn.RMSNorm``: fp32 statistics, ``x * rsqrt(mean(x^2)+eps) * scale``."""
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * scale.float()
    return y.to(x.dtype)


def causal_conv1d(x: Tensor, w: Tensor, bias: Optional[Tensor], silu: bool) -> Tensor:
    """Depthwise causal conv over time.  ``x (B,L,C)``, ``w (C,W)`` (flax layout
    ``(features, width)``, tap ``W-1`` hits the current token), ``bias (C,)``."""
    Bsz, L, Cn = x.shape
    W = w.shape[1]
    xt = F.pad(x.transpose(1, 2), (W - 1, 0))
    y = F.conv1d(xt, w.to(x.dtype)[:, None, :], None, groups=Cn).transpose(1, 2)
    if bias is not None:
        y = y + bias.to(x.dtype)
    return F.silu(y) if silu else y


def gelu_tanh(x: Tensor) -> Tensor:
    """``jax.nn.gelu`` default (tanh approximation)."""
    return F.gelu(x, approximate="tanh")


def safe_l2norm(x: Tensor, eps2: float) -> Tensor:
    xf = x.float()
    return (xf * torch.rsqrt((xf * xf).sum(-1, keepdim=True) + eps2)).to(x.dtype)


def label_smoothed_ce(logits: Tensor, labels: Tensor, label_smoothing: float) -> Tuple[Tensor, Tensor]:
    """Reference chunk CE (reference `optimizer.py:244-281`): returns (sum_loss, sum_mask).

    ``loss = nll*(sp - sn) - sn*sum(log_probs)`` with ``sp = 1-ls`` and
    ``sn = ls/(V-1)``; labels ``-100`` are masked out.
    """
    V = logits.shape[-1]
    lf = logits.float()
    lf = torch.nan_to_num(lf, nan=0.0, posinf=1e4, neginf=-1e4).clamp(-1e4, 1e4)
    logp = torch.log_softmax(lf, -1)
    safe = labels.clamp(0, V - 1)
    nll = -logp.gather(-1, safe[:, None].long()).squeeze(-1)
    if label_smoothing > 0:
        sp, sn = 1.0 - label_smoothing, label_smoothing / (V - 1)
        loss = nll * (sp - sn) - sn * logp.sum(-1)
    else:
        loss = nll
    mask = (labels != -100).float()
    return torch.where(mask > 0, loss, torch.zeros_like(loss)).sum(), mask.sum()


def rope_cos_sin(seq_len: int, dim: int, device=None, dtype=torch.float32):
    inv = 1.0 / (10000 ** (torch.arange(0, dim, 2, device=device, dtype=torch.float32)[: dim // 2] / dim))
    t = torch.arange(seq_len, device=device, dtype=torch.float32)
    fr = torch.outer(t, inv)
    emb = torch.cat([fr, fr], -1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def apply_rope(x: Tensor, cos: Tensor, sin: Tensor) -> Tensor:
    d = x.shape[-1]
    x1, x2 = x[..., : d // 2], x[..., d // 2:]
    rot = torch.cat([-x2, x1], -1)
    return x * cos.to(x.dtype) + rot * sin.to(x.dtype)


def causal_attention(q: Tensor, k: Tensor, v: Tensor, sm_scale: float) -> Tensor:
    """``(B,H,L,D)`` causal softmax attention in fp32."""
    s = torch.einsum("bhqd,bhkd->bhqk", q.float(), k.float()) * sm_scale
    L = q.shape[2]
    mask = torch.ones(L, L, dtype=torch.bool, device=q.device).tril()
    s = s.masked_fill(~mask, -1e9)
    return torch.einsum("bhqk,bhkd->bhqd", s.softmax(-1), v.float()).to(q.dtype)


def grouped_ffn(x_sorted: Tensor, group_sizes, w1: Tensor, w2: Tensor, w3: Optional[Tensor], act: str):
    """Per-expert FFN over token rows sorted by expert.  ``w1 (E,d,F)``, ``w2 (E,F,d)``,
    ``w3 (E,d,F)`` for SwiGLU.  Rows of expert ``e`` are contiguous."""
    outs = []
    start = 0
    sizes = [int(s) for s in group_sizes]
    for e, n in enumerate(sizes):
        xe = x_sorted[start:start + n]
        h = sanitize(xe @ w1[e], 1e3)
        if act == "swiglu":
            h = F.silu(h) * sanitize(xe @ w3[e], 1e3)
        else:
            h = gelu_tanh(h)
        outs.append(sanitize(h @ w2[e], 1e3))
        start += n
    return torch.cat(outs, 0) if outs else x_sorted.new_zeros(0, w2.shape[-1])


def newton_schulz3(g: Tensor, steps: int = 3, eps: float = 1e-4) -> Tensor:
    """Reference Muon orthogonalisation (reference `optimizer.py:53-77`)."""
    if g.ndim == 3:
        nrm = torch.linalg.vector_norm(g, dim=(-2, -1), keepdim=True)
        nrm = torch.where(nrm < eps, torch.ones_like(nrm), nrm)
        X = g / nrm
        for _ in range(steps):
            X = 1.5 * X - 0.5 * (X @ X.transpose(-1, -2) @ X)
            X = torch.nan_to_num(X, nan=0.0, posinf=0.0, neginf=0.0)
    else:
        nrm = torch.linalg.vector_norm(g)
        nrm = torch.where(nrm < eps, torch.ones_like(nrm), nrm)
        X = g / nrm
        for _ in range(steps):
            X = 1.5 * X - 0.5 * (X @ X.T @ X)
            X = torch.nan_to_num(X, nan=0.0, posinf=0.0, neginf=0.0)
    return X


def flops_gdn_chunked(B: int, L: int, H: int, D: int, C: int) -> float:
    """Matmul FLOPs of one chunked GDN forward (used for scan TFLOP/s)."""
    nc = L // C
    per_chunk = (2 * C * C * D * 2            # Aqk, Akk
                 + 2 * C * C * D * 2          # w_pseudo, u
                 + 2 * C * D * D * 3          # w h, q h, k^T v
                 + 2 * C * C * D)             # Aqk v_new
    return float(B * H * nc * per_chunk)


def flops_ssd_chunked(B: int, L: int, H: int, P: int, N: int, C: int) -> float:
    nc = L // C
    per_chunk = (2 * C * C * N + 2 * C * C * P      # CB, y_diag
                 + 2 * C * P * N * 2)               # state_end, y_off
    return float(B * H * nc * per_chunk)


__all__ = [n for n in dir() if not n.startswith("_")]
_ = math
