"""Operator entry points used by the models.

Two implementations exist for every op:

* ``"cuda"``  -- the product path: hand-written sm_100a kernels in
  ``atomic_ai_hybrid_b200/csrc`` (loaded from the in-tree extension
  ``_ahb_cuda*.so``).  Selected by default for CUDA tensors.  If the extension
  is missing on a machine with a GPU the op raises instead of falling back.
* ``"eager"`` -- plain PyTorch (``ops.reference``), the unfused baseline of the
  benchmark and the only path for CPU tensors.

``set_impl("eager")`` forces the baseline on the GPU (used by ``bench.py --impl
eager``); ``set_impl("cuda")`` is the default.
"""
from __future__ import annotations

import contextlib
import os
from typing import Optional

import torch
import torch.nn.functional as F

from . import reference as R

_IMPL = os.environ.get("AHB_IMPL", "cuda")


def set_impl(name: str) -> None:
    global _IMPL
    assert name in ("cuda", "eager"), name
    _IMPL = name


def get_impl() -> str:
    return _IMPL


@contextlib.contextmanager
def impl(name: str):
    old = _IMPL
    set_impl(name)
    try:
        yield
    finally:
        set_impl(old)


def use_cuda(*tensors: torch.Tensor) -> bool:
    """True when the CUDA kernels must run for these tensors."""
    if _IMPL != "cuda":
        return False
    return all(t.is_cuda for t in tensors if isinstance(t, torch.Tensor))


def _k():
    from . import kernels
    return kernels


# ---------------------------------------------------------------- gradient guards
class _GradSanitize(torch.autograd.Function):
    """Identity forward; backward clips the cotangent to ``+-clip`` and replaces
    non-finite values (reference ``make_grad_sanitizer``, `model.py:192-217`)."""

    @staticmethod
    def forward(ctx, x, clip, tag):
        ctx.clip, ctx.tag = clip, tag
        return x.view_as(x)

    @staticmethod
    def backward(ctx, g):
        if ctx.tag is not None:
            from ..utils.diag import DIAG
            DIAG.grad_fixed(ctx.tag, g)
        if g.is_cuda and _IMPL == "cuda":
            return _k().sanitize(g, ctx.clip), None, None
        return R.sanitize(g, ctx.clip), None, None


def grad_sanitize(x: torch.Tensor, clip: float = 1e3, tag: Optional[str] = None) -> torch.Tensor:
    """``tag``: report a non-finite incoming gradient as ``[BWD-FIX]`` (``utils.diag``)."""
    if not torch.is_grad_enabled() or not x.requires_grad:
        return x
    return _GradSanitize.apply(x, clip, tag)


def sanitize(x: torch.Tensor, clip: float) -> torch.Tensor:
    if use_cuda(x):
        return _k().sanitize_fwd(x, clip)
    return R.sanitize(x, clip)


# ---------------------------------------------------------------- dense / norm
def linear(x: torch.Tensor, kernel: torch.Tensor, bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``x @ kernel (+ bias)`` in the dtype of ``x`` (cuBLAS for plain GEMMs)."""
    w = kernel if kernel.dtype == x.dtype else kernel.to(x.dtype)
    if bias is not None:
        b = bias if bias.dtype == x.dtype else bias.to(x.dtype)
        return torch.addmm(b, x.reshape(-1, x.shape[-1]), w).view(*x.shape[:-1], w.shape[-1])
    return torch.matmul(x, w)


def rmsnorm(x: torch.Tensor, scale: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    if use_cuda(x):
        return _k().rmsnorm(x, scale, eps)
    return R.rmsnorm(x, scale, eps)


def conv1d(x: torch.Tensor, w: torch.Tensor, b: Optional[torch.Tensor], silu: bool = True,
           clip: Optional[float] = None) -> torch.Tensor:
    """Depthwise causal conv (+bias, +SiLU, optional output clamp)."""
    if use_cuda(x):
        return _k().conv1d(x, w, b, silu, clip)
    y = R.causal_conv1d(x, w, b, silu)
    return y.clamp(-clip, clip) if clip is not None else y


# ---------------------------------------------------------------- sequence mixers
def gdn2(q, k, v, w, b, g, scale: float = 1.0, chunk: int = 64, h0=None, return_final: bool = False):
    """GDN-2 chunked delta rule; ``(B,L,H,D)`` inputs, per-channel gates.  ``h0`` (B,H,D,D)
    is the state before the first token; ``return_final`` returns ``(o, h_final)``."""
    if use_cuda(q):
        return _k().gdn2(q, k, v, w, b, g, scale, chunk, h0=h0, return_final=return_final)
    o, hf = R.gdn2_chunked(q, k, v, g, b, w, scale, chunk, h0=h0, checkpoint_chunks=True)
    return (o, hf) if return_final else o


def ssd(dt, A, Bm, Cm, x, chunk: int = 64, state0=None, return_final: bool = False):
    """Mamba2 SSD; ``dt, x (B,L,H,P)``, ``A (H,)``, ``B, C (B,L,N)``.  ``state0`` (B,H,P,N)
    is the state before the first token; ``return_final`` returns ``(y, s_final)``."""
    if use_cuda(x):
        return _k().ssd(dt, A, Bm, Cm, x, chunk, state0=state0, return_final=return_final)
    y, sf = R.ssd_chunked(dt, A, Bm, Cm, x, chunk, state0=state0, checkpoint_chunks=True)
    return (y, sf) if return_final else y


def attention(q, k, v, sm_scale: float) -> torch.Tensor:
    """Causal attention on ``(B,H,L,D)``."""
    if use_cuda(q):
        return _k().attention(q, k, v, sm_scale)
    if q.dtype == torch.float32 or q.dtype == torch.float64:
        return R.causal_attention(q, k, v, sm_scale)
    return F.scaled_dot_product_attention(q, k, v, is_causal=True, scale=sm_scale)


# ---------------------------------------------------------------- MoE
def grouped_ffn(x_sorted, group_sizes, w1, w2, w3, act: str, group_sizes_cpu=None):
    if use_cuda(x_sorted):
        return _k().grouped_ffn(x_sorted, group_sizes, w1, w2, w3, act)
    sizes = group_sizes_cpu if group_sizes_cpu is not None else group_sizes.tolist()
    dt = x_sorted.dtype
    return R.grouped_ffn(x_sorted, sizes, w1.to(dt), w2.to(dt), None if w3 is None else w3.to(dt), act)


# ---------------------------------------------------------------- loss
def cross_entropy(hidden: torch.Tensor, labels: torch.Tensor, weight: torch.Tensor,
                  label_smoothing: float, chunk: int = 2048):
    """Label-smoothed CE of ``hidden @ weight^T`` (tied LM head, ``weight (V,d)``).

    Returns ``(sum_loss, sum_mask)``; the logits are never materialised for the
    whole batch (chunks of ``chunk`` tokens, recomputed in backward)."""
    h = hidden.reshape(-1, hidden.shape[-1])
    lab = labels.reshape(-1)
    if use_cuda(h):
        return _k().cross_entropy(h, lab, weight, label_smoothing)
    import torch.utils.checkpoint as ckpt

    wd = weight.to(h.dtype)

    def piece(hc, lc):
        logits = (hc @ wd.t()).float()
        return R.label_smoothed_ce(logits, lc, label_smoothing)

    tot = h.new_zeros((), dtype=torch.float32)
    cnt = h.new_zeros((), dtype=torch.float32)
    for s in range(0, h.shape[0], chunk):
        if torch.is_grad_enabled():
            a, c = ckpt.checkpoint(piece, h[s:s + chunk], lab[s:s + chunk], use_reentrant=False)
        else:
            a, c = piece(h[s:s + chunk], lab[s:s + chunk])
        tot = tot + a
        cnt = cnt + c
    return tot, cnt
