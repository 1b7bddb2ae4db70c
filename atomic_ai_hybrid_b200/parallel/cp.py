"""Context parallelism for the recurrent layers: every rank holds a contiguous segment of
each sequence (positions ``[r L / W, (r + 1) L / W)``) and the mixers pass what crosses the
segment boundaries.

The reference scales sequence length only through its chunked scans on one device
(`atomic_ops/kernel_d_pipeline.py:94-158`, `atomic_ops/kernel_mamba2_c_interchunk.py:83`);
this module splits the sequence over ranks instead, exactly:

* **scans** (GDN-2 and SSD) are affine in their initial state ``h0``:
  ``h_end = T h0 + S`` and ``out(h0, v) = out(0, v) + out(h0, 0)``.  Each rank runs its
  segment from ``h0 = 0`` (giving ``out(0, v)`` and ``S``), runs the transition ``T``
  (GDN-2: the segment from ``h0 = I`` with zero values, a ``D x D`` map per head; SSD:
  per-channel decay factors, from ``h0 = 1`` with zero inputs, floored per chunk as the
  reference floors them), all-gathers the ``(T, S)`` pairs, folds the ones of the earlier
  ranks into its incoming state ``h_in`` and adds ``out(h_in, 0)``.  The value clips of the
  scans (``+-1e4``) are the only non-linear parts; while they are inactive the result equals
  the single-rank one.
* **causal convolutions** read the last ``width - 1`` inputs of the previous rank (a halo);
* **MLA** gathers the latent of every position (``d_latent`` wide), recomputes K and V for
  the whole sequence and attends from its own queries with the causal offset.

Everything is differentiable through an all-gather whose backward is an all-to-all (NCCL
or gloo), so the backward passes the state and halo gradients back along the same paths.  Every rank
builds the same graph (the first rank weights its incoming state and halo by zero rather
than skipping them), so the backward issues the same collectives in the same order on all
ranks.  Per-token
work (norms, MoE, embedding, loss) is local, as with data parallelism; every parameter is
replicated, and its gradient is summed over the ranks like a data-parallel one.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.distributed as dist


class _Gather(torch.autograd.Function):
    """All-gather whose backward sums each rank's gradients of every slot back to the slot's
    owner with one all-to-all over contiguous buffers (the gradients that reach it can be
    strided views, e.g. of a concatenation)."""

    @staticmethod
    def forward(ctx, group, world, t):
        ctx.group, ctx.world = group, world
        t = t.contiguous()
        out = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(out, t, group=group)
        return tuple(out)

    @staticmethod
    def backward(ctx, *grads):
        send = torch.stack([g.contiguous() for g in grads])
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=ctx.group)
        return None, None, recv.sum(0)


class CPGroup:
    def __init__(self, world: int, rank: int, group: Optional[dist.ProcessGroup] = None):
        self.world, self.rank, self.group = world, rank, group
        self.seq_len: Optional[int] = None

    # ------------------------------------------------------------ layout
    def set_seq(self, L: int) -> None:
        if L % self.world:
            raise ValueError(f"sequence length {L} does not split over {self.world} context-parallel ranks")
        self.seq_len = L

    @property
    def seg(self) -> Tuple[int, int]:
        n = self.seq_len // self.world
        return self.rank * n, (self.rank + 1) * n

    def local_time(self, t: torch.Tensor) -> torch.Tensor:
        lo, hi = self.seg
        return t[:, lo:hi]

    # ------------------------------------------------------------ collectives (differentiable)
    def gather(self, t: torch.Tensor):
        return _Gather.apply(self.group, self.world, t)

    def gather_time(self, x: torch.Tensor) -> torch.Tensor:
        """``(B, L / W, ...)`` -> ``(B, L, ...)``."""
        return torch.cat(self.gather(x), 1)

    def prev_rows(self, x: torch.Tensor, n: int) -> torch.Tensor:
        """The last ``n`` time rows of the previous rank's ``x`` (zeros on rank 0).

        Every rank builds the same graph (rank 0 scales its pick by zero instead of skipping
        it), so the backward runs the collectives in the same order everywhere."""
        tails = self.gather(x[:, -n:])
        return tails[(self.rank - 1) % self.world] * (1.0 if self.rank > 0 else 0.0)

    # ------------------------------------------------------------ layer pieces
    def causal_conv(self, conv, x: torch.Tensor, w: torch.Tensor, b, **kw) -> torch.Tensor:
        """``conv`` (a causal depthwise conv over dim 1) of the whole sequence, this segment's
        outputs: the inputs are prefixed by the previous segment's last ``width - 1`` rows."""
        halo = w.shape[1] - 1
        xx = torch.cat([self.prev_rows(x, halo), x], 1)
        return conv(xx, w, b, **kw)[:, halo:]

    def _fold(self, Ts, Ss, apply):
        """Incoming state of this rank: ``h <- T_j h + S_j`` over the ranks before it.  The
        loop runs over every rank with 0/1 weights, so all ranks build the same graph."""
        h = torch.zeros_like(Ss[0])
        for j in range(self.world):
            c = 1.0 if j < self.rank else 0.0
            h = c * (apply(Ts[j], h) + Ss[j]) + (1.0 - c) * h
        return h

    def gdn2_scan(self, q, k, v, g, b, w, scale: float, chunk: int):
        """This segment's GDN-2 output given the states of the segments before it: the local
        scan from zero (output ``o0``, final state ``S``), the segment's state transfer ``T``
        (the final state of a scan from the identity with ``v = 0``: ``h -> T h``), the
        incoming state folded over the earlier ranks, and the output of that state carried
        through the segment (``v = 0``).  On CUDA the three scans are the sm_100a kernels
        with their initial-state inputs and gradients."""
        from .. import ops
        o0, S = ops.gdn2(q, k, v, w, b, g, scale, chunk, return_final=True)
        B, L, H, D = q.shape
        eye = torch.eye(D, dtype=torch.float32, device=q.device).expand(B, H, D, D).contiguous()
        zv = torch.zeros_like(v)
        _, T = ops.gdn2(q, k, zv, w, b, g, scale, chunk, h0=eye, return_final=True)
        Ts, Ss = self.gather(T), self.gather(S)
        h_in = self._fold(Ts, Ss, lambda Tj, h: Tj @ h)
        oc = ops.gdn2(q, k, zv, w, b, g, scale, chunk, h0=h_in)
        return o0 + oc

    def ssd_scan(self, dt, A, Bm, Cm, x, chunk: int):
        """Mamba2 SSD of this segment given the earlier segments' states (as ``gdn2_scan``;
        the transfer of a segment is a per-(head, channel) decay, the final state of a scan
        from ones with ``x = 0``)."""
        from .. import ops
        y0, S = ops.ssd(dt, A, Bm, Cm, x, chunk, return_final=True)
        zx = torch.zeros_like(x)
        _, T = ops.ssd(dt, A, Bm, Cm, zx, chunk, state0=torch.ones_like(S), return_final=True)
        Ts, Ss = self.gather(T), self.gather(S)
        h_in = self._fold(Ts, Ss, lambda Tj, h: Tj * h)
        yc = ops.ssd(dt, A, Bm, Cm, zx, chunk, state0=h_in)
        return y0 + yc


def get_cp() -> Optional[CPGroup]:
    from .context import get_parallel_context
    cp = getattr(get_parallel_context(), "cp", None)
    return cp if cp is not None and cp.world > 1 else None


def init_context_parallel(device: Optional[torch.device] = None, cp_size: Optional[int] = None) -> CPGroup:
    """Context-parallel groups of ``cp_size`` consecutive ranks (all ranks by default; the
    ``world / cp_size`` groups are data-parallel replicas that read different batches);
    install this rank's group in the parallel context.  Every parameter is replicated on
    every rank, so gradients and batch statistics are summed / averaged over all ranks
    (each rank holds different tokens: its segment of its replica's sequences)."""
    from .context import ParallelContext, set_parallel_context
    world, rank = dist.get_world_size(), dist.get_rank()
    size = cp_size or world
    if world % size:
        raise ValueError(f"{world} ranks do not split into context-parallel groups of {size}")
    group = None
    if size < world:
        for start in range(0, world, size):  # every rank creates every group, in order
            g = dist.new_group(list(range(start, start + size)))
            if start <= rank < start + size:
                group = g
    cp = CPGroup(size, rank % size, group)
    ctx = ParallelContext(dp_group=None, dp_world=world)
    ctx.cp = cp
    set_parallel_context(ctx)
    return cp
