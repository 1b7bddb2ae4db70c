"""Autograd wrappers around the sm_100a kernels of ``_ahb_cuda``.

Weight gradients are accumulated directly into the fp32 gradient store when a
parameter carries ``_ahb_grad_acc`` (set by ``FlatParamStore``): the kernel adds
into the accumulator and autograd sees no gradient for that weight, so no bf16
weight-gradient tensor is materialised per micro-step.  Without an accumulator
(plain module use) the wrapper returns an ordinary gradient.
"""
from __future__ import annotations

import math
import os
from typing import Optional

import torch
import torch.nn.functional as F

from . import reference as R
from ._ext import ext
from ..utils.diag import DIAG


def _acc_for(p: Optional[torch.Tensor]):
    """(accumulator, owned_here) for a parameter: the store's fp32 view if any,
    else a fresh zero fp32 buffer whose content becomes the returned gradient."""
    if p is None:
        return None, False
    acc = getattr(p, "_ahb_grad_acc", None)
    if acc is not None:
        return acc, True
    return torch.zeros(p.shape, dtype=torch.float32, device=p.device), False


def _ret_grad(p, acc, direct):
    if p is None or not p.requires_grad or direct:
        return None
    return acc.to(p.dtype)


# ----------------------------------------------------------------- sanitize
def sanitize(g: torch.Tensor, clip: float) -> torch.Tensor:
    if g.dtype not in (torch.bfloat16, torch.float32):
        return R.sanitize(g, clip)
    return ext().sanitize(g, clip)


class _SanitizeFwd(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, clip):
        y = ext().sanitize(x, clip)
        ctx.save_for_backward(x)
        ctx.clip = clip
        return y

    @staticmethod
    def backward(ctx, g):
        (x,) = ctx.saved_tensors
        # d clip: pass where |x| < clip (NaN/inf inputs get no gradient)
        mask = x.abs() < ctx.clip
        return g * mask, None


def sanitize_fwd(x: torch.Tensor, clip: float) -> torch.Tensor:
    if x.dtype not in (torch.bfloat16, torch.float32):
        return R.sanitize(x, clip)
    if torch.is_grad_enabled() and x.requires_grad:
        return _SanitizeFwd.apply(x, clip)
    return ext().sanitize(x, clip)


# ----------------------------------------------------------------- RMSNorm
class _RMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, scale, eps):
        shp = x.shape
        y, rstd = ext().rmsnorm_fwd(x.reshape(-1, shp[-1]), scale, eps)
        ctx.save_for_backward(x, scale, rstd)
        return y.view(shp)

    @staticmethod
    def backward(ctx, dy):
        x, scale, rstd = ctx.saved_tensors
        acc, direct = _acc_for(scale) if ctx.needs_input_grad[1] else (None, False)
        d = x.shape[-1]
        dx = ext().rmsnorm_bwd(dy.reshape(-1, d), x.reshape(-1, d), scale, rstd, acc)
        return dx.view(x.shape), _ret_grad(scale, acc, direct), None


def rmsnorm(x, scale, eps):
    return _RMSNorm.apply(x, scale, eps)


# ----------------------------------------------------------------- conv1d
class _Conv1d(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, b, silu, clip):
        y = ext().conv1d_fwd(x, w, b, silu, clip)
        ctx.save_for_backward(x, w, b)
        ctx.silu, ctx.clip = silu, clip
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w, b = ctx.saved_tensors
        wacc, wdir = _acc_for(w)
        bacc, bdir = _acc_for(b) if b is not None else (None, False)
        dx = ext().conv1d_bwd(x, w, b, dy.to(x.dtype), ctx.silu, ctx.clip, wacc, bacc)
        return dx, _ret_grad(w, wacc, wdir), _ret_grad(b, bacc, bdir), None, None


def conv1d(x, w, b, silu=True, clip=None):
    if x.stride(-1) != 1 or x.stride(0) != x.shape[1] * x.stride(1):
        x = x.contiguous()
    return _Conv1d.apply(x, w, b, silu, 0.0 if clip is None else float(clip))


# ----------------------------------------------------------------- embedding
class _Embed(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ids, table, dtype):
        out = ext().embedding_fwd(ids.reshape(-1), table, dtype)
        ctx.save_for_backward(ids)
        ctx.table = table
        return out.view(*ids.shape, table.shape[1])

    @staticmethod
    def backward(ctx, dout):
        (ids,) = ctx.saved_tensors
        table = ctx.table
        acc, direct = _acc_for(table)
        ext().embedding_bwd_(ids.reshape(-1), dout.reshape(-1, table.shape[1]), acc)
        return None, _ret_grad(table, acc, direct), None


def embedding(ids, table, dtype):
    return _Embed.apply(ids, table, dtype)


# ----------------------------------------------------------------- not yet native
# Keep the chunk intermediates of the scans for the backward (default) instead of
# recomputing them there, as the reference's B6 backward does (`atomic_ops/
# kernel_trainable_B6.py:104-109`); AHB_SCAN_RECOMPUTE=1 trades the memory back.
SCAN_RECOMPUTE = os.environ.get("AHB_SCAN_RECOMPUTE", "0") == "1"


class _GDN2(torch.autograd.Function):
    """sm_100a chunked GDN-2 (head dim 128, chunk 64): 2 launches forward; the
    backward runs 4 launches on the saved chunk intermediates (WY factors, scores,
    per-chunk states), or 6 when it recomputes them.  ``h0`` (B,H,128,128), the state
    before the first token, and the returned final state are differentiable (reference
    initial-state path: `atomic_ops/kernel_trainable_B6.py:187-193`)."""

    @staticmethod
    def forward(ctx, q, k, v, g, b, w, scale, h0, want_final):
        bf = torch.bfloat16
        q, k, v, b, w = (t.to(bf).contiguous() for t in (q, k, v, b, w))
        g = g.float().contiguous()
        h0 = h0.float().contiguous() if h0 is not None else None
        keep = any(ctx.needs_input_grad) and not SCAN_RECOMPUTE
        hf = None
        if keep:
            o, *inter = ext().gdn_fwd_train(q, k, v, g, b, w, scale, h0, want_final)
            if want_final:
                hf = inter.pop()
        else:
            outs = ext().gdn_fwd(q, k, v, g, b, w, scale, want_final, h0)
            o, hf = outs[0], (outs[1] if want_final else None)
            inter = []
        ctx.n_inter = len(inter)
        ctx.has_h0 = h0 is not None
        ctx.save_for_backward(q, k, v, g, b, w, *((h0,) if h0 is not None else ()), *inter)
        ctx.scale = scale
        ctx.want_final = want_final
        return (o, hf) if want_final else o

    @staticmethod
    def backward(ctx, do, dhf=None):
        q, k, v, g, b, w, *rest = ctx.saved_tensors
        h0 = rest.pop(0) if ctx.has_h0 else None
        inter = rest
        want_dh0 = ctx.has_h0 and ctx.needs_input_grad[7]
        dhf = dhf.float().contiguous() if dhf is not None else None
        if inter:
            grads = ext().gdn_bwd_saved(q, k, v, g, b, w, do.contiguous(), ctx.scale, inter, dhf, want_dh0)
        else:
            grads = ext().gdn_bwd(q, k, v, g, b, w, do.contiguous(), ctx.scale, h0, dhf, want_dh0)
        dq, dk, dv, dg, db, dw = grads[:6]
        return dq, dk, dv, dg, db, dw, None, (grads[6] if want_dh0 else None), None


_WARNED = set()


def _unsupported(what: str) -> None:
    if what not in _WARNED:
        _WARNED.add(what)
        print(f"[atomic_ai_hybrid_b200] {what}: shape not covered by the sm_100a kernel; "
              f"using the PyTorch chunked path", flush=True)


def gdn2(q, k, v, w, b, g, scale, chunk, h0=None, return_final=False):
    """``(B,L,H,128)`` GDN-2 with per-channel gates; ``chunk`` is fixed at 64 in the kernel
    (results do not depend on the chunk length).  ``h0`` (B,H,128,128) is the state before
    the first token (zero when None); ``return_final`` also returns the fp32 state after the
    last one, as ``(o, h_final)``; both carry gradients.  Other head dims or lengths that are
    not a multiple of 64 run the PyTorch chunked path."""
    if q.shape[-1] != 128 or q.shape[1] % 64:
        _unsupported(f"gdn2 D={q.shape[-1]} L={q.shape[1]}")
        o, hf = R.gdn2_chunked(q, k, v, g, b, w, scale, chunk, h0=h0, checkpoint_chunks=True)
        return (o, hf) if return_final else o
    return _GDN2.apply(q, k, v, g, b, w, float(scale), h0, bool(return_final))


class _SSD(torch.autograd.Function):
    """sm_100a Mamba2 SSD (head dim 64, d_state 128, chunk 64): 2 launches forward
    (chunk kernel, state recurrence); the backward reuses the forward's per-chunk states and
    intra-chunk outputs (4 launches: reverse state-gradient recurrence, chunk backward, two
    group sums) or recomputes them (6).  ``s0`` (B,H,64,128), the state before the first
    token, and the returned final state are differentiable (reference initial-state path:
    `atomic_ops/kernel_mamba2_trainable_B6.py:137-155`)."""

    @staticmethod
    def forward(ctx, dt, A, Bm, Cm, x, s0, want_final):
        bf = torch.bfloat16
        dt, Bm, Cm, x = (t.to(bf).contiguous() for t in (dt, Bm, Cm, x))
        A = A.float().contiguous()
        s0 = s0.float().contiguous() if s0 is not None else None
        sf = None
        if any(ctx.needs_input_grad) and not SCAN_RECOMPUTE or s0 is not None or want_final:
            y, *saved = ext().ssd_fwd_train(x, dt, A, Bm, Cm, s0, want_final)
            if want_final:
                sf = saved.pop()
            if not any(ctx.needs_input_grad) or SCAN_RECOMPUTE:
                saved = []
        else:
            y = ext().ssd_fwd(x, dt, A, Bm, Cm)
            saved = []
        ctx.has_s0 = s0 is not None
        ctx.save_for_backward(dt, A, Bm, Cm, x, *((s0,) if s0 is not None else ()), *saved)
        return (y, sf) if want_final else y

    @staticmethod
    def backward(ctx, dy, dsf=None):
        dt, A, Bm, Cm, x, *st = ctx.saved_tensors
        s0 = st.pop(0) if ctx.has_s0 else None
        want_ds0 = ctx.has_s0 and ctx.needs_input_grad[5]
        dsf = dsf.float().contiguous() if dsf is not None else None
        saved = st if st else [None] * 4
        grads = ext().ssd_bwd(x, dt, A, Bm, Cm, dy.contiguous(), *saved, s0, dsf, want_ds0)
        dx, ddt, dA, dB, dC = grads[:5]
        return ddt, dA, dB.to(Bm.dtype), dC.to(Cm.dtype), dx, (grads[5] if want_ds0 else None), None


def ssd(dt, A, Bm, Cm, x, chunk, state0=None, return_final=False):
    """``dt, x (B,L,H,64)``, ``A (H,)``, ``B, C (B,L,128)``; chunk fixed at 64 in the kernel.
    ``state0`` (B,H,64,128) is the state before the first token (zero when None);
    ``return_final`` also returns the fp32 state after the last one, as ``(y, s_final)``;
    both carry gradients.  Other head dims / state sizes run the PyTorch chunked path."""
    if x.shape[-1] != 64 or Bm.shape[-1] != 128 or x.shape[1] % 64:
        _unsupported(f"ssd P={x.shape[-1]} N={Bm.shape[-1]} L={x.shape[1]}")
        y, sf = R.ssd_chunked(dt, A, Bm, Cm, x, chunk, state0=state0, checkpoint_chunks=True)
        return (y, sf) if return_final else y
    return _SSD.apply(dt, A, Bm, Cm, x, state0, bool(return_final))


class _Attention(torch.autograd.Function):
    """Causal flash attention (``attention.cu``): forward keeps O and the row
    log-sum-exp; backward recomputes P per key tile."""

    @staticmethod
    def forward(ctx, q, k, v, scale):
        o, lse = ext().attn_fwd(q, k, v, scale)
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.scale = scale
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse = ctx.saved_tensors
        dq, dk, dv = ext().attn_bwd(q, k, v, o, do, lse, ctx.scale)
        return dq, dk, dv, None


def attention(q, k, v, sm_scale):
    """Causal attention on ``(B, H, L, D)`` bf16 with D in {64, 96, 128}; other
    head dims or dtypes use PyTorch's scaled_dot_product_attention."""
    if q.dtype == torch.bfloat16 and q.shape[-1] in (64, 96, 128):
        bf = torch.bfloat16
        return _Attention.apply(q.to(bf).contiguous(), k.to(bf).contiguous(), v.to(bf).contiguous(), float(sm_scale))
    _unsupported(f"attention D={q.shape[-1]} dtype={q.dtype}")
    return F.scaled_dot_product_attention(q, k, v, is_causal=True, scale=sm_scale)


def grouped_ffn(x_sorted, group_sizes, w1, w2, w3, act):
    dt = x_sorted.dtype
    return R.grouped_ffn(x_sorted, group_sizes.tolist(), w1.to(dt), w2.to(dt),
                         None if w3 is None else w3.to(dt), act)


# rows per backward chunk of the LM head: the chunk's bf16 dlogits (rows x V) are the head's only
# vocabulary-wide buffer (8192 x 50304: 824 MB); the forward stores no logits at all
CE_CHUNK_ROWS = int(os.environ.get("AHB_CE_CHUNK_ROWS", "8192"))


class _FusedCE(torch.autograd.Function):
    """Tied LM head + label-smoothed CE that never stores the logits: the tcgen05 head GEMM
    reduces each (row, 256-column vocabulary tile) to online-softmax partials in its epilogue
    and a combine kernel forms the row log-sum-exp and the loss; the backward recomputes the
    logits tile by tile into dlogits for one row chunk at a time, followed by the dh and fp32
    weight-gradient GEMMs (reference `optimizer.py:244-312`, chunked cross entropy)."""

    @staticmethod
    def forward(ctx, h, labels, weight, ls):
        wb = weight if weight.dtype == torch.bfloat16 else weight.to(torch.bfloat16)
        wb = wb.contiguous()
        hb = h.to(torch.bfloat16).contiguous()
        lab = labels.to(torch.long).contiguous()
        sum_loss, count, lse = ext().ce_online_fwd(hb, wb, lab, ls)
        ctx.save_for_backward(hb, lab, lse)
        ctx.weight, ctx.wb, ctx.ls = weight, wb, ls
        ctx.hdtype = h.dtype
        return sum_loss.reshape(()), count.reshape(())

    @staticmethod
    def backward(ctx, g_loss, g_count):
        hb, lab, lse = ctx.saved_tensors
        acc, direct = _acc_for(ctx.weight)
        dh = ext().ce_online_bwd(hb, ctx.wb, lab, lse, ctx.ls, g_loss.reshape(1), acc, CE_CHUNK_ROWS)
        return dh.to(ctx.hdtype), None, _ret_grad(ctx.weight, acc, direct), None


def cross_entropy(h, labels, weight, label_smoothing):
    """``(sum_loss, sum_mask)`` of the tied LM head; see ``_FusedCE``."""
    return _FusedCE.apply(h, labels, weight, float(label_smoothing))


# ----------------------------------------------------------------- fused layer glue
def row_fusable(d: int) -> bool:
    """Rows handled by the fused row kernels: D/8 threads with 16-byte accesses."""
    return d % 256 == 0 and d <= 8192


class _AddRMSNorm(torch.autograd.Function):
    """``xo = sanitize(x + delta, clip)``, ``y = rmsnorm(xo) * scale``; the
    backward optionally sanitizes the delta gradient (grad sanitizer on a sublayer
    output)."""

    @staticmethod
    def forward(ctx, x, delta, scale, clip, eps, sanitize_delta_grad, stats):
        xo, y, rstd = ext().add_rmsnorm_fwd(x, delta.contiguous(), scale, clip, eps, stats)
        ctx.save_for_backward(xo, scale, rstd)
        ctx.clip, ctx.sdg = clip, sanitize_delta_grad
        return xo, y

    @staticmethod
    def backward(ctx, gxo, gy):
        xo, scale, rstd = ctx.saved_tensors
        acc, direct = _acc_for(scale) if ctx.needs_input_grad[2] else (None, False)
        if gy is None:
            gy = torch.zeros_like(xo)
        dx, dd = ext().add_rmsnorm_bwd(gy, gxo, xo, scale, rstd, ctx.clip, ctx.sdg, acc)
        return dx, dd, _ret_grad(scale, acc, direct), None, None, None, None


def add_rmsnorm(x, delta, scale, clip: float, eps: float = 1e-6, sanitize_delta_grad: bool = False,
                diag_tag: Optional[str] = None):
    """``diag_tag``: fold ``max |x + delta|`` and a non-finite-delta flag into the step
    diagnostics (``utils.diag``) from inside the kernel."""
    stats = None
    if diag_tag is not None:
        from ..utils.diag import DIAG
        stats = DIAG.residual_pair(diag_tag, x.device)
    return _AddRMSNorm.apply(x, delta, scale, clip, eps, sanitize_delta_grad, stats)


class _NormGate(torch.autograd.Function):
    """``clamp(rmsnorm(x) * scale * silu(clamp(z, +-zclip)), +-oclip)``."""

    @staticmethod
    def forward(ctx, x, z, scale, eps, zclip, oclip):
        y, rstd = ext().norm_gate_fwd(x, z, scale, eps, zclip, oclip)
        ctx.save_for_backward(x, z, scale, rstd)
        ctx.zclip, ctx.oclip = zclip, oclip
        return y

    @staticmethod
    def backward(ctx, dy):
        x, z, scale, rstd = ctx.saved_tensors
        acc, direct = _acc_for(scale) if ctx.needs_input_grad[2] else (None, False)
        dx, dz = ext().norm_gate_bwd(dy, x, z, scale, rstd, ctx.zclip, ctx.oclip, acc)
        return dx, dz.view(z.shape), _ret_grad(scale, acc, direct), None, None, None


def norm_gate(x, z, scale, eps: float = 1e-6, zclip: float = math.inf, oclip: float = math.inf):
    return _NormGate.apply(x.contiguous(), z, scale, eps, zclip, oclip)


class _GDNGates(torch.autograd.Function):
    """Per-channel GDN-2 gates: ``sigmoid`` erase / write gates and the decay
    ``g = clamp(nan_to_num(-exp(clamp(a)) * softplus(f)), +-1e3)`` (fp32)."""

    @staticmethod
    def forward(ctx, bp, wp, fp, decay_a, Dh):
        bg, wg, g = ext().gdn_gates_fwd(bp, wp, fp, decay_a, Dh)
        ctx.save_for_backward(bg, wg, fp, decay_a)
        ctx.Dh = Dh
        return bg, wg, g

    @staticmethod
    def backward(ctx, dbg, dwg, dg):
        bg, wg, fp, decay_a = ctx.saved_tensors
        dbg = torch.zeros_like(bg) if dbg is None else dbg
        dwg = torch.zeros_like(wg) if dwg is None else dwg
        dg = torch.zeros(bg.shape, dtype=torch.float32, device=bg.device) if dg is None else dg
        acc, direct = _acc_for(decay_a) if ctx.needs_input_grad[3] else (None, False)
        dbp, dwp, dfp, acc_out = ext().gdn_gates_bwd(dbg, dwg, dg, bg, wg, fp, decay_a, ctx.Dh, acc)
        return dbp, dwp, dfp, _ret_grad(decay_a, acc_out, direct), None


def gdn_gates(bp, wp, fp, decay_a, Dh: int):
    return _GDNGates.apply(bp.contiguous(), wp.contiguous(), fp.contiguous(), decay_a, Dh)


class _L2NormHeads(torch.autograd.Function):
    """Per-head L2 normalisation (head dim 128) followed by the gradient sanitizer."""

    @staticmethod
    def forward(ctx, x):
        y, rn = ext().l2norm_heads_fwd(x)
        ctx.save_for_backward(x, rn)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, rn = ctx.saved_tensors
        return ext().l2norm_heads_bwd(dy, x, rn)


def l2norm_heads(x):
    return _L2NormHeads.apply(x.contiguous())


class _DtAct(torch.autograd.Function):
    @staticmethod
    def forward(ctx, u):
        ctx.save_for_backward(u)
        return ext().dt_act_fwd(u)

    @staticmethod
    def backward(ctx, ddt):
        (u,) = ctx.saved_tensors
        return ext().dt_act_bwd(ddt, u)


def dt_act(u):
    """Mamba2 ``clamp(softplus(u), 0.01, 1)``."""
    return _DtAct.apply(u.contiguous())


# ----------------------------------------------------------------- dense projections
_ADDMM_F32 = None  # whether cuBLAS accumulates bf16 products straight into fp32 (probed once)


def _rows(t):
    """``t`` as the dense GEMM reads it: unit column stride and 16-byte-aligned rows (a column slice
    of a wider buffer stays a view; anything else is copied)."""
    if t.stride(-1) == 1 and t.stride(0) % 8 == 0 and t.data_ptr() % 16 == 0:
        return t
    return t.contiguous()


def _dense_ok(x2, w) -> bool:
    """Shapes and types the tcgen05 dense GEMM takes for ``x2 (M, K) @ w (K, N)``."""
    return (x2.is_cuda and x2.dtype == torch.bfloat16 and w.dtype == torch.bfloat16 and w.dim() == 2
            and w.shape[0] % 64 == 0 and w.shape[1] % 32 == 0)


def _wgrad_acc(acc, x2, dy2):
    """``acc (in, out) fp32 += x2^T dy2`` with bf16 inputs: the tcgen05 K-grouped GEMM adds into
    the fp32 accumulator in its epilogue; shapes it does not cover run one library GEMM with
    beta = 1 and fp32 output."""
    global _ADDMM_F32
    if (x2.is_cuda and x2.dtype == torch.bfloat16 and dy2.dtype == torch.bfloat16 and acc.dtype == torch.float32
            and acc.is_contiguous() and x2.shape[1] % 128 == 0 and dy2.shape[1] % 32 == 0):
        ext().dense_wgrad(_rows(x2), _rows(dy2), acc)
        return
    _unsupported(f"dense weight gradient in={x2.shape[1]} out={dy2.shape[1]}")
    if _ADDMM_F32 is not False:
        try:
            torch.addmm(acc, x2.t(), dy2, out_dtype=torch.float32, out=acc)
            _ADDMM_F32 = True
            return
        except (RuntimeError, TypeError):
            _ADDMM_F32 = False
    acc.add_((x2.t() @ dy2).float())


def bias_grad(b, dy2):
    """Gradient of a bias from ``dy2 (M, N)``: added straight into the fp32 gradient
    store by a column-sum kernel when the bias has an accumulator (returns None),
    else returned as an fp32 tensor."""
    acc = getattr(b, "_ahb_grad_acc", None) if b is not None else None
    if (acc is not None and dy2.is_cuda and dy2.dtype == torch.bfloat16 and dy2.shape[1] % 8 == 0
            and acc.dtype == torch.float32 and acc.numel() == dy2.shape[1]):
        ext().bias_grad_acc(_rows(dy2), acc.view(-1))
        return None
    return dy2.sum(0, dtype=torch.float32)


class _MultiLinear(torch.autograd.Function):
    """Several projections of one input, ``y_i = x W_i (+ b_i)``, on the tcgen05 dense GEMM
    (CTA pairs, bias added in the epilogue; reference `model.py:405-427,575-613`).  The
    backward accumulates ``dx = sum_i dy_i W_i^T`` in one buffer (each GEMM after the first
    adds the previous value in its epilogue) and adds the weight gradients of store-backed
    matrices straight into their fp32 accumulators from the GEMM epilogue.  Shapes the kernel
    does not cover (in % 64, out % 32) run library GEMMs."""

    @staticmethod
    def forward(ctx, x, n, *wb):
        ws, bs = wb[:n], wb[n:]
        x2 = x.reshape(-1, x.shape[-1])
        outs = []
        for w, b in zip(ws, bs):
            wc = w if w.dtype == x.dtype else w.to(x.dtype)
            if _dense_ok(x2, wc):
                y = ext().dense_fwd(_rows(x2), wc.contiguous(), b)
            else:
                _unsupported(f"dense projection in={wc.shape[0]} out={wc.shape[1]}")
                y = torch.addmm(b.to(x.dtype), x2, wc) if b is not None else torch.mm(x2, wc)
            outs.append(y.view(*x.shape[:-1], w.shape[1]))
        ctx.save_for_backward(x, *ws)
        ctx.n, ctx.has_b = n, [b is not None for b in bs]
        ctx.bs = list(bs)
        return tuple(outs)

    @staticmethod
    def backward(ctx, *dys):
        x, *ws = ctx.saved_tensors
        b_params = ctx.bs
        x2 = x.reshape(-1, x.shape[-1])
        dx = None
        dws, dbs = [], []
        for w, dy, hb in zip(ws, dys, ctx.has_b):
            if dy is None:
                dws.append(None)
                dbs.append(None)
                continue
            dy2 = dy.reshape(-1, dy.shape[-1]).to(x.dtype)
            wc = w if w.dtype == x.dtype else w.to(x.dtype)
            if ctx.needs_input_grad[0]:
                if dy2.is_cuda and dy2.dtype == torch.bfloat16 and wc.dtype == torch.bfloat16 and \
                        wc.shape[1] % 64 == 0 and wc.shape[0] % 32 == 0:
                    first = dx is None
                    if first:
                        dx = torch.empty(x2.shape, dtype=x.dtype, device=x.device)
                    ext().dense_dgrad(_rows(dy2), wc.contiguous(), dx, not first)
                elif dx is None:
                    _unsupported(f"dense input gradient in={wc.shape[0]} out={wc.shape[1]}")
                    dx = torch.mm(dy2, wc.t())
                else:
                    torch.addmm(dx, dy2, wc.t(), out=dx)
            acc = getattr(w, "_ahb_grad_acc", None)
            if acc is not None and w.dtype != torch.float32:
                _wgrad_acc(acc.view(w.shape), x2, dy2)
                dws.append(None)
            else:
                g32 = torch.zeros(w.shape, dtype=torch.float32, device=x.device)
                _wgrad_acc(g32, x2, dy2)
                dws.append(g32.to(w.dtype))
            dbs.append(bias_grad(b_params[len(dbs)], dy2) if hb else None)
        if dx is not None:
            dx = dx.view(x.shape)
        return (dx, None, *dws, *dbs)


def linear_multi(x, pairs):
    """``[(kernel (in, out), bias or None), ...]`` -> the projections of ``x``."""
    ws = [w for w, _ in pairs]
    bs = [b for _, b in pairs]
    return _MultiLinear.apply(x, len(pairs), *ws, *bs)


class _SwiGLU(torch.autograd.Function):
    """Shared-expert gate ``silu(a) * b`` on bf16 for the SwiGLU configurations (the
    reference's shared expert, `atomic_ops/moe_gmm.py:396-399`, is the GELU variant): one
    kernel each way, fp32 inside with one rounding per output."""

    @staticmethod
    def forward(ctx, a, b):
        ctx.save_for_backward(a, b)
        return ext().swiglu_fwd(a, b)

    @staticmethod
    def backward(ctx, dh):
        a, b = ctx.saved_tensors
        da, db = ext().swiglu_bwd(dh, a, b)
        return da, db


def swiglu(a, b):
    if (a.is_cuda and a.dtype == torch.bfloat16 and b.dtype == torch.bfloat16 and a.shape == b.shape
            and a.is_contiguous() and b.is_contiguous() and a.numel() % 8 == 0):
        return _SwiGLU.apply(a, b)
    return F.silu(a) * b


class _Router(torch.autograd.Function):
    """Fused cosine router: returns the differentiable (gate, sum_t softmax(l),
    sum_t lse^2) and the non-differentiable (top_idx, expert counts, statistics)."""

    @staticmethod
    def forward(ctx, x, kn, temp, bias, noise, k):
        logits, cosv, rn, top, gate, psum, scal, counts = ext().router_fwd(x, kn, temp, bias, noise, k)
        ctx.save_for_backward(x, kn, temp, logits, cosv, rn, top, gate)
        ctx.mark_non_differentiable(top, counts, scal)
        return gate, psum, scal[0:1].clone(), top, counts, scal

    @staticmethod
    def backward(ctx, dgate, dpsum, dlse, _dtop, _dcounts, _dscal):
        x, kn, temp, logits, cosv, rn, top, gate = ctx.saved_tensors
        dgate = torch.zeros_like(gate) if dgate is None else dgate
        dpsum = torch.zeros(logits.shape[1], device=x.device) if dpsum is None else dpsum
        dx, dkn, dtemp = ext().router_bwd(x, kn, temp, logits, cosv, rn, top, gate, dgate, dpsum, dlse)
        return dx, dkn, dtemp.view(temp.shape), None, None, None


def router_supported(d: int, E: int, k: int) -> bool:
    return bool(ext().router_supported(d, E, k))


def router(x, kn, temp, bias, noise, k: int):
    """``x (T, d)`` bf16, ``kn (d, E)`` unit-column router kernel, ``temp (1,)``."""
    return _Router.apply(x.contiguous(), kn, temp, bias, noise, k)


class _SourceMix(torch.autograd.Function):
    """``sum_i softmax_i(scale <q, k_i>) s_i`` per token (BlockDAR source softmax)."""

    @staticmethod
    def forward(ctx, scale, n, q, *ks_ss):
        ks, ss = list(ks_ss[:n]), list(ks_ss[n:])
        out, wts = ext().source_mix_fwd(q, ks, ss, scale)
        ctx.save_for_backward(q, wts, *ks, *ss)
        ctx.scale, ctx.n = scale, n
        return out

    @staticmethod
    def backward(ctx, g):
        q, wts, *rest = ctx.saved_tensors
        n = ctx.n
        res = ext().source_mix_bwd(g, q, rest[:n], rest[n:], wts, ctx.scale)
        return (None, None, res[0], *res[1:])


def source_mix(q, ks, ss, scale: float):
    """``q (..., dl)``, ``ks`` n tensors like ``q``, ``ss`` n tensors ``(..., d)``; bf16.
    Returns ``None`` where the kernel does not apply (the caller uses PyTorch ops)."""
    n = len(ss)
    if (n == 0 or n > 32 or q.dtype != torch.bfloat16 or any(t.dtype != torch.bfloat16 for t in ss)
            or torch.cuda.is_current_stream_capturing()):
        return None
    bf = torch.bfloat16
    ks = [k.to(bf).contiguous() for k in ks]
    ss = [s.contiguous() for s in ss]
    return _SourceMix.apply(float(scale), n, q.to(bf).contiguous(), *ks, *ss)


def gdn2_layer(mod, x):
    if x.dtype == torch.bfloat16 and mod.d_head == 128 and row_fusable(mod.cfg.d_model):
        return _gdn2_layer_fused(mod, x)
    return _gdn2_layer_composed(mod, x)


class _TPNorm(torch.autograd.Function):
    """RMSNorm over the full width of a head-split activation, gated like ``norm_gate``
    when ``z`` is given (the mixer output norms ``out_norm`` / ``ssm_out_norm``, reference
    `model.py:652` and `model.py:520`, with the heads split over the tensor-parallel group).  Each
    direction is two kernel passes with one all-reduce of a per-row fp32 sum between them:
    the sum of squares in the forward, the dot of the normalised input with its gradient
    in the backward.  Nothing else crosses the group."""

    @staticmethod
    def forward(ctx, x, z, scale, eps, d_full, tp, zclip, oclip):
        import torch.distributed as dist
        ss = ext().tp_norm_sumsq(x)
        dist.all_reduce(ss, group=tp.group)
        y, rstd = ext().tp_norm_fwd(x, z, scale, ss, eps, 1.0 / d_full, zclip, oclip)
        ctx.save_for_backward(x, z, scale, rstd)
        ctx.tp, ctx.inv, ctx.zclip, ctx.oclip = tp, 1.0 / d_full, zclip, oclip
        return y

    @staticmethod
    def backward(ctx, dy):
        import torch.distributed as dist
        x, z, scale, rstd = ctx.saved_tensors
        dy = dy.contiguous()
        acc, direct = _acc_for(scale) if ctx.needs_input_grad[2] else (None, False)
        dz, dot = ext().tp_norm_bwd_dot(dy, x, z, scale, rstd, ctx.zclip, ctx.oclip, acc)
        dist.all_reduce(dot, group=ctx.tp.group)
        dx = ext().tp_norm_bwd_dx(dy, x, z, scale, rstd, dot, ctx.inv, ctx.zclip, ctx.oclip)
        return (dx, None if z is None else dz.view(z.shape), _ret_grad(scale, acc, direct), None, None, None, None,
                None)


def tp_norm(x, z, scale, eps: float, d_full: int, tp, zclip: float = math.inf, oclip: float = math.inf):
    """``clamp(rmsnorm_group(x) * scale [* silu(clamp(z, +-zclip))], +-oclip)`` for bf16 rows
    of ``x.shape[-1] % 256 == 0`` channels, ``d_full`` channels over the group."""
    return _TPNorm.apply(x.contiguous(), z, scale, eps, d_full, tp, zclip, oclip)


def _out_norm_gate(mod_cfg_d, o, z, scale, zclip=math.inf, oclip=math.inf):
    """Gated RMSNorm of a mixer output; over all heads of the tensor-parallel group
    when the heads are split (all-reduced statistics)."""
    from ..parallel.tp import get_tp, tp_norm_gate
    tp = get_tp()
    if tp is not None:
        if o.is_cuda and o.dtype == torch.bfloat16 and z.dtype == torch.bfloat16 and row_fusable(o.shape[-1]):
            return tp_norm(o, z, scale, 1e-6, mod_cfg_d, tp, zclip=zclip, oclip=oclip)
        return tp_norm_gate(o, z, scale, 1e-6, mod_cfg_d, tp, zclip=zclip, oclip=oclip)
    return norm_gate(o, z, scale, 1e-6, zclip=zclip, oclip=oclip)


def _gdn2_layer_fused(mod, x):
    H, D = mod.n_heads, mod.d_head
    qp, kp, vp, bp, wp, fp, og = mod.projections(x)
    Bsz, L, dl = qp.shape
    q = conv1d(qp, mod.q_conv_w, mod.q_conv_b, True)
    k = conv1d(kp, mod.k_conv_w, mod.k_conv_b, True)
    v = conv1d(vp, mod.v_conv_w, mod.v_conv_b, True, 50.0)
    q = l2norm_heads(q.view(Bsz, L, H, D))
    k = l2norm_heads(k.view(Bsz, L, H, D))
    bg, wg, g = gdn_gates(bp, wp, fp, mod.decay_a, D)
    shp = (Bsz, L, H, D)
    DIAG.stage("GDN2", "q", q)
    DIAG.stage("GDN2", "k", k)
    DIAG.stage("GDN2", "v", v)
    DIAG.stage("GDN2", "g", g)
    o = gdn2(q, k, v.view(shp), wg.view(shp), bg.view(shp), g.view(shp), 1.0, mod.cfg.gdn_chunk)
    DIAG.stage("GDN2", "o", o)
    o = _out_norm_gate(mod.cfg.d_model, o.reshape(Bsz, L, dl).to(x.dtype), og, mod.out_norm.scale, zclip=1e2)
    return mod.out_projection(o)


def _gdn2_layer_composed(mod, x):
    H, D = mod.n_heads, mod.d_head
    qp, kp, vp, bp, wp, fp, og = mod.projections(x)
    Bsz, L, dl = qp.shape
    q = conv1d(qp, mod.q_conv_w, mod.q_conv_b, True)
    k = conv1d(kp, mod.k_conv_w, mod.k_conv_b, True)
    v = conv1d(vp, mod.v_conv_w, mod.v_conv_b, True, 50.0)
    q = R.safe_l2norm(q.view(Bsz, L, H, D), 1e-12)
    k = R.safe_l2norm(k.view(Bsz, L, H, D), 1e-12)
    from .. import ops
    q = ops.grad_sanitize(q)
    k = ops.grad_sanitize(k)
    v = v.view(Bsz, L, H, D)
    bg = torch.sigmoid(bp).view(Bsz, L, H, D)
    wg = torch.sigmoid(wp).view(Bsz, L, H, D)
    f = fp.view(Bsz, L, H, D).float()
    g = -torch.exp(mod.decay_a.float().clamp(-20.0, 20.0))[None, None, :, None] * F.softplus(f)
    g = torch.nan_to_num(g, nan=0.0, posinf=0.0, neginf=-20.0).clamp(-1e3, 1e3)
    og = og.clamp(-1e2, 1e2)
    o = gdn2(q, k, v, wg, bg, g, 1.0, mod.cfg.gdn_chunk).reshape(Bsz, L, dl)
    from ..parallel.tp import get_tp, tp_rmsnorm
    tp = get_tp()
    if tp is not None:
        o = tp_rmsnorm(o, mod.out_norm.scale, 1e-6, mod.cfg.d_model, tp).to(o.dtype)
    else:
        o = rmsnorm(o, mod.out_norm.scale, 1e-6)
    return mod.out_projection(o * F.silu(og))


def mamba2_layer(mod, x):
    Hs = mod.n_heads
    xz = mod.in_projection(x)
    Bsz, L, two_dil = xz.shape
    dil = two_dil // 2
    P = dil // Hs
    fused = x.dtype == torch.bfloat16 and row_fusable(dil)
    x_bc, res = xz[..., :dil], xz[..., dil:]
    DIAG.stage("MAMBA2", "in_proj", xz)
    x_conv = conv1d(x_bc, mod.conv_w, mod.conv_b, True)
    DIAG.stage("MAMBA2", "x_conv", x_conv)
    A = -torch.exp(mod.A_log.float().clamp(-20.0, 20.0))
    xin = mod.bc_input(x_bc)
    Bm, Cm, dtp = linear_multi(xin, [(m.kernel, m.bias) for m in (mod.B_proj, mod.C_proj, mod.dt_proj)])
    dt = dt_act(dtp) if fused else F.softplus(dtp).clamp(1e-2, 1.0)
    DIAG.stage("MAMBA2", "dt", dt)
    y = ssd(dt.view(Bsz, L, Hs, P), A, Bm.clamp(-1e3, 1e3), Cm.clamp(-1e3, 1e3), x_conv.view(Bsz, L, Hs, P),
            mod.cfg.ssd_chunk)
    y = y.reshape(Bsz, L, dil).to(x_bc.dtype)
    DIAG.stage("MAMBA2", "ssd_y", y)
    if fused:
        return mod.out_projection(_out_norm_gate(mod.cfg.d_inner, y, res, mod.ssm_out_norm.scale, oclip=3e2))
    from ..parallel.tp import get_tp, tp_rmsnorm
    tp = get_tp()
    if tp is not None:
        y = tp_rmsnorm(y, mod.ssm_out_norm.scale, 1e-6, mod.cfg.d_inner, tp).to(y.dtype)
    else:
        y = rmsnorm(y, mod.ssm_out_norm.scale, 1e-6)
    out = (y * F.silu(res)).clamp(-3e2, 3e2)
    return mod.out_projection(out)


class _MoE(torch.autograd.Function):
    """Dropless top-k routed experts + combine on the tcgen05 grouped GEMM.

    Forward: route positions -> gather -> fused up-projection (SwiGLU/GELU in the
    epilogue) -> down-projection -> gated combine with the shared-expert output.
    Backward: combine backward -> dH with the activation backward in the epilogue ->
    dX (both up-projections in one K-concatenated GEMM) -> weight gradients added
    straight into the fp32 gradient store."""

    @staticmethod
    def forward(ctx, x, top_idx, gate, w1, w2, w3, shared, swiglu):
        bf = torch.bfloat16
        xs_ = x.to(bf).contiguous()
        w1b, w2b = w1.to(bf).contiguous(), w2.to(bf).contiguous()
        w3b = None if w3 is None else w3.to(bf).contiguous()
        outs = ext().moe_fwd(xs_, top_idx, gate.float(), w1b, w2b, w3b,
                             None if shared is None else shared.to(bf), swiglu)
        out, pos, off, row_src, xs, a1, a3, h, ys = outs
        ctx.save_for_backward(gate, pos, off, row_src, xs, a1, a3, h, ys)
        ctx.w = (w1, w2, w3, w1b, w2b, w3b)
        ctx.swiglu = swiglu
        ctx.has_shared = shared is not None
        return out

    @staticmethod
    def backward(ctx, dout):
        gate, pos, off, row_src, xs, a1, a3, h, ys = ctx.saved_tensors
        w1, w2, w3, w1b, w2b, w3b = ctx.w
        a1c, d1 = _acc_for(w1)
        a2c, d2 = _acc_for(w2)
        a3c, d3 = _acc_for(w3) if w3 is not None else (None, False)
        dx, dgate = ext().moe_bwd(dout.contiguous(), gate.float(), w1b, w2b, w3b, pos, off, row_src, xs, a1, a3, h,
                                  ys, a1c, a2c, a3c, ctx.swiglu)
        dshared = dout if ctx.has_shared else None
        return (dx, None, dgate, _ret_grad(w1, a1c, d1), _ret_grad(w2, a2c, d2),
                None if w3 is None else _ret_grad(w3, a3c, d3), dshared, None)


def moe_forward(flat, top_idx, gate, w1, w2, w3, shared, act):
    """Combined MoE output ``sanitize(shared + sum_j gate_j * expert_j(x), 1e3)`` in bf16."""
    return _MoE.apply(flat, top_idx, gate, w1, w2, w3, shared, act == "swiglu")


def gemm_error() -> int:
    """Error word of the tcgen05 kernels (0 = no timed-out wait since the last reset)."""
    return int(ext().gemm_error())


def newton_schulz3(g, steps: int = 3, eps: float = 1e-4):
    """Muon orthogonalisation (reference `optimizer.py:53-77`): ``steps`` Newton-Schulz steps
    X <- 1.5 X - 0.5 X X^T X on the tcgen05 grouped GEMM (``muon_ns``: bf16 operands, fp32
    accumulation, X itself kept in fp32, non-finite entries zeroed after every step).

    The step commutes with transposition, so the Gram matrix is taken on the shorter side
    (r x r): X X^T for a wide matrix, X^T X (K-grouped GEMM) for several tall ones, and a single
    tall matrix runs as its transpose.  The matrices of a 3-D tensor
    (the experts) are the groups of the same two launches per step.  A shorter side that is not a
    multiple of 128 (or a longer one not of 64) runs the fp32 PyTorch iteration instead."""
    if not g.is_cuda or g.ndim not in (2, 3):
        return R.newton_schulz3(g, steps, eps)
    m = g if g.ndim == 3 else g.unsqueeze(0)
    tall = m.shape[1] > m.shape[2]
    r, c = (m.shape[2], m.shape[1]) if tall else (m.shape[1], m.shape[2])
    if r % 128 or c % 64:
        return R.newton_schulz3(g, steps, eps)
    if tall and m.shape[0] >= 2 and c % 128 == 0:
        # several tall matrices (the experts' up-projections): X^T X from the K-grouped GEMM,
        # no transposed copies
        X = m.float()
        nrm = torch.linalg.vector_norm(X, dim=(-2, -1), keepdim=True)
        X = (X / torch.where(nrm < eps, torch.ones_like(nrm), nrm)).contiguous()
        for e0 in range(0, X.shape[0], 192):
            part = X[e0:e0 + 192]
            if part.shape[0] >= 2:
                ext().muon_ns_tall(part, steps)
            else:  # a lone last matrix (already of norm 1) runs as its transpose
                part.copy_(newton_schulz3(part[0], steps, eps).unsqueeze(0))
        return X.reshape(g.shape)
    X = (m.transpose(1, 2) if tall else m).float()
    nrm = torch.linalg.vector_norm(X, dim=(-2, -1), keepdim=True)
    X = (X / torch.where(nrm < eps, torch.ones_like(nrm), nrm)).contiguous()
    for e0 in range(0, X.shape[0], 192):  # the grouped GEMM takes at most 192 groups
        ext().muon_ns(X[e0:e0 + 192], steps)
    out = X.transpose(1, 2) if tall else X
    return out.reshape(g.shape)


# ----------------------------------------------------------------- fused optimizer
_WD = {"muon": 0.01, "lion": 0.1, "adamw_decay": 0.01, "adamw_nodecay": 0.0, "frozen": 0.0}
_ORDER = ("muon", "lion", "adamw_decay", "adamw_nodecay", "frozen")


def _optim_table(opt):
    if getattr(opt, "_segs", None) is not None:
        return
    from ..optim.schedule import LABEL_ID, diag_group_of, path_key
    st = opt.store
    rows, gs, nblocks = [], [], 0
    chunk = 4096
    for s in opt.owned:
        key = path_key(s.name)
        flags = (1 if s.fp32 else 0) | (2 if "router_temp" in key else 0) | (4 if "expert_bias" in key else 0) \
            | (8 if s.param.requires_grad else 0)
        brow = opt.bias_index(s) if "expert_bias" in key else 0
        rows.append([s.offset - st.lo, s.coff, s.numel, LABEL_ID[s.label], opt.group_idx[diag_group_of(s.name)],
                     flags, brow, 0])
        gs.append(s.grad_scale)
        nblocks += (s.numel + chunk - 1) // chunk
    dev = st.device.index if st.device.index is not None else torch.cuda.current_device()
    opt._segs, opt._cstart = ext().optim_make_table(torch.tensor(rows, dtype=torch.int64),
                                                    torch.tensor(gs, dtype=torch.float32), dev)
    opt._nblocks = nblocks


def optim_prepare(opt, inv, red):
    """One pass over the owned gradients: average, non-finite flags, both norms, was_clipped."""
    _optim_table(opt)
    st = opt.store
    redd = torch.zeros(2, dtype=torch.float64, device=st.device)
    flags = torch.zeros(8, dtype=torch.int32, device=st.device)
    peers = getattr(opt, "peers", None)
    ext().optim_prepare(opt._segs, opt._cstart, opt._nblocks, st.grad[st.lo:st.hi], st.master, float(inv), redd, flags,
                        peers[0] if peers else None, st.lo)
    red[0:2] = redd.float()
    red[2:] = flags.float()


def optim_apply(opt, lrs, coef, frac):
    """Per-label update + clip + hooks + compute-copy write, one kernel.  With
    ``opt.peers`` set, prepare sums the owned gradient slice over the peers'
    buffers and apply writes the compute copies of every peer."""
    st = opt.store
    peers = getattr(opt, "peers", None)
    t = opt.count + 1
    lr = [float(lrs[k]) for k in _ORDER]
    wd = [_WD[k] for k in _ORDER]
    ext().optim_apply(opt._segs, opt._cstart, opt._nblocks, st.master, opt.m, opt.v, st.grad[st.lo:st.hi],
                      coef.reshape(1).float().contiguous(), st.compute, frac, lr, wd, 1.0 - 0.9 ** t,
                      1.0 - 0.999 ** t, peers[1] if peers else None)


_ = math
