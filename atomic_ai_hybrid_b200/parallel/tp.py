"""Tensor parallelism with sequence parallelism over the GPUs of one node.

The reference has no tensor parallelism: it runs GSPMD FSDP + DP on a 1-D mesh
(`train_setup.py:361-365,415-436`).  The long-context configuration of the
benchmark splits the heads of every sequence mixer over the ranks of a node, which
this module provides, Megatron-style with sequence parallelism:

* the residual stream, the RMSNorms, the MoE, the embedding and the loss work on a
  contiguous block of the flattened ``(batch x sequence)`` tokens: rank ``r`` holds
  rows ``[r * T / W, (r + 1) * T / W)``;
* a sequence mixer (GDN-2, Mamba2, MLA) gathers the token rows of its input
  (all-gather over tokens) and computes its ``1 / W`` of the heads over the full
  sequences; its output projection is row-parallel and the partial sums go back to
  token blocks with a reduce-scatter;
* column-parallel weights hold output features ``[r n / W, (r + 1) n / W)`` of every
  block of their output (Mamba2's ``in_proj`` has two blocks, ``x_bc`` and the gate);
  row-parallel weights hold the same rows of their input; per-channel and per-head
  vectors follow their channels;
* an RMSNorm over the full width of a head-split activation (GDN ``out_norm``, Mamba2
  ``ssm_out_norm``, MLA ``attn_out_norm``) all-reduces the per-row sum of squares.

Each rank's loss is the mean over its own tokens (as a data-parallel rank's), so
gradients of replicated parameters are summed over every rank and scaled like
data-parallel ones, and the gradients of split parameters arrive complete through
the backward of the collectives.

Two implementations of the collectives:

* ``torch.distributed`` (NCCL, or gloo on the CPU) - the baseline and the CPU path;
* ``parallel.tp_peer.PeerTP`` on CUDA: token rows move between NVLink peer buffers
  (CUDA IPC); the all-gather runs on the copy engines while the projections of the
  rows already present proceed, and the forward row-parallel projection is one
  tcgen05 GEMM whose epilogue stores each partial tile straight into the receive
  buffer of the rank that owns those rows.
"""
from __future__ import annotations

from typing import List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist


def split_range(n: int, world: int, rank: int) -> Tuple[int, int]:
    if n % world:
        raise ValueError(f"{n} does not split over {world} tensor-parallel ranks")
    k = n // world
    return rank * k, (rank + 1) * k


def shard_tensor(full: torch.Tensor, dim: int, parts: int, world: int, rank: int) -> torch.Tensor:
    """The slice of ``full`` that rank ``rank`` holds: ``dim`` is cut into ``parts``
    equal blocks and every block into ``world`` pieces; piece ``rank`` of each block,
    concatenated in block order."""
    n = full.shape[dim]
    if n % parts:
        raise ValueError(f"dimension {dim} of size {n} is not {parts} equal blocks")
    blk = n // parts
    lo, hi = split_range(blk, world, rank)
    pieces = [full.narrow(dim, b * blk + lo, hi - lo) for b in range(parts)]
    return torch.cat(pieces, dim) if parts > 1 else pieces[0]


def unshard_tensors(shards: Sequence[torch.Tensor], dim: int, parts: int) -> torch.Tensor:
    """Inverse of ``shard_tensor`` over all ranks' pieces (in rank order)."""
    if parts == 1:
        return torch.cat(list(shards), dim)
    blocks = []
    for b in range(parts):
        for s in shards:
            k = s.shape[dim] // parts
            blocks.append(s.narrow(dim, b * k, k))
    return torch.cat(blocks, dim)


def mark_shard(p: torch.Tensor, dim: int, parts: int = 1) -> torch.Tensor:
    """Tag a parameter as this rank's tensor-parallel piece (see ``shard_tensor``)."""
    p._ahb_tp_shard = (dim, parts)
    return p


def shard_spec(p: torch.Tensor) -> Optional[Tuple[int, int]]:
    return getattr(p, "_ahb_tp_shard", None)


# ------------------------------------------------------------ raw collectives
def _ag0(x: torch.Tensor, group, world: int) -> torch.Tensor:
    out = x.new_empty((world * x.shape[0],) + tuple(x.shape[1:]))
    dist.all_gather_into_tensor(out, x.contiguous(), group=group)
    return out


def _rs0(x: torch.Tensor, group, world: int) -> torch.Tensor:
    out = x.new_empty((x.shape[0] // world,) + tuple(x.shape[1:]))
    dist.reduce_scatter_tensor(out, x.contiguous(), group=group)
    return out


class _GatherTokens(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, tp):
        ctx.tp = tp
        return tp.impl_gather_tokens(x)

    @staticmethod
    def backward(ctx, g):
        return ctx.tp.impl_scatter_tokens(g.contiguous()), None


class _ScatterTokens(torch.autograd.Function):
    @staticmethod
    def forward(ctx, y, tp):
        ctx.tp = tp
        return tp.impl_scatter_tokens(y)

    @staticmethod
    def backward(ctx, g):
        return ctx.tp.impl_gather_tokens(g.contiguous()), None


class _AllReduce(torch.autograd.Function):
    """Sum over the ranks; the backward sums the gradients (every rank's output
    feeds its own loss terms)."""

    @staticmethod
    def forward(ctx, x, tp):
        ctx.tp = tp
        y = x.clone()
        dist.all_reduce(y, group=tp.group)
        return y

    @staticmethod
    def backward(ctx, g):
        g = g.clone()
        dist.all_reduce(g, group=ctx.tp.group)
        return g, None


class _GatherFeatures(torch.autograd.Function):
    """``(T, n / W)`` pieces -> ``(T, n)``; the backward reduce-scatters along features."""

    @staticmethod
    def forward(ctx, x, tp):
        ctx.tp = tp
        T, dl = x.shape
        g = _ag0(x, tp.group, tp.world)  # (W*T, dl)
        return g.view(tp.world, T, dl).permute(1, 0, 2).reshape(T, tp.world * dl)

    @staticmethod
    def backward(ctx, g):
        tp = ctx.tp
        T, n = g.shape
        dl = n // tp.world
        gt = g.view(T, tp.world, dl).permute(1, 0, 2).contiguous().view(tp.world * T, dl)
        return _rs0(gt, tp.group, tp.world), None


class TPGroup:
    """The tensor-parallel ranks of one node and the state of one forward pass (the
    global ``(batch, sequence)`` shape that the mixers restore after a gather)."""

    def __init__(self, world: int, rank: int, group: Optional[dist.ProcessGroup] = None,
                 peer=None):
        self.world, self.rank, self.group = world, rank, group
        self.peer = peer  # PeerTP: NVLink peer-memory collectives (CUDA)
        self.batch_shape: Optional[Tuple[int, int]] = None

    # ------------------------------------------------------------ token layout
    def set_batch(self, bsz: int, seq: int) -> None:
        if (bsz * seq) % self.world:
            raise ValueError(f"{bsz} x {seq} tokens do not split over {self.world} tensor-parallel ranks")
        self.batch_shape = (bsz, seq)

    @property
    def local_rows(self) -> int:
        b, l = self.batch_shape
        return b * l // self.world

    def local_tokens(self, t: torch.Tensor) -> torch.Tensor:
        """``(B, L, ...)`` -> this rank's block ``(1, B L / W, ...)`` of the flattened tokens."""
        flat = t.reshape((-1,) + tuple(t.shape[2:]))
        n = flat.shape[0] // self.world
        return flat[self.rank * n:(self.rank + 1) * n].unsqueeze(0)

    # ------------------------------------------------------------ collectives (autograd)
    def gather_tokens(self, x: torch.Tensor) -> torch.Tensor:
        """``(..., d)`` local rows -> ``(B, L, d)`` rows of all ranks."""
        d = x.shape[-1]
        full = _GatherTokens.apply(x.reshape(-1, d), self)
        return full.view(*self.batch_shape, d)

    def scatter_tokens(self, y: torch.Tensor) -> torch.Tensor:
        """``(B, L, d)`` partial sums -> ``(1, B L / W, d)`` summed local rows."""
        d = y.shape[-1]
        return _ScatterTokens.apply(y.reshape(-1, d), self).unsqueeze(0)

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        return _AllReduce.apply(x, self)

    def gather_features(self, x: torch.Tensor) -> torch.Tensor:
        shp = x.shape
        out = _GatherFeatures.apply(x.reshape(-1, shp[-1]), self)
        return out.view(*shp[:-1], out.shape[-1])

    # ------------------------------------------------------------ fused layer edges
    def gather_linear(self, x: torch.Tensor, pairs: List[Tuple[torch.Tensor, Optional[torch.Tensor]]]):
        """Projections of the gathered token rows: ``[gather(x) W_i (+ b_i)]`` as
        ``(B, L, n_i)`` tensors.  The peer path overlaps the row transfers with the
        projections of the rows already present."""
        if self.peer is not None and self.peer.usable(x):
            return self.peer.gather_linear(x, pairs, self.batch_shape)
        xf = self.gather_tokens(x)
        from .. import ops
        if ops.use_cuda(xf) and xf.dtype == torch.bfloat16:
            from ..ops import kernels as K
            return list(K.linear_multi(xf, pairs))
        return [ops.linear(xf, w, b) for w, b in pairs]

    def linear_scatter(self, o: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        """Row-parallel projection ``o W`` summed over the ranks and returned as this
        rank's token rows ``(1, B L / W, n)``."""
        if self.peer is not None and self.peer.usable(o):
            return self.peer.linear_scatter(o, w)
        from .. import ops
        if ops.use_cuda(o) and o.dtype == torch.bfloat16:
            from ..ops import kernels as K
            y = K.linear_multi(o, [(w, None)])[0]
        else:
            y = ops.linear(o, w)
        return self.scatter_tokens(y)

    # ------------------------------------------------------------ implementations
    def impl_gather_tokens(self, x: torch.Tensor) -> torch.Tensor:
        if self.peer is not None and self.peer.usable(x):
            return self.peer.all_gather_rows(x)
        return _ag0(x, self.group, self.world)

    def impl_scatter_tokens(self, y: torch.Tensor) -> torch.Tensor:
        if self.peer is not None and self.peer.usable(y):
            return self.peer.reduce_scatter_rows(y)
        return _rs0(y, self.group, self.world)

    def close(self) -> None:
        if self.peer is not None:
            self.peer.close()
            self.peer = None


def get_tp() -> Optional[TPGroup]:
    from .context import get_parallel_context
    tp = get_parallel_context().tp
    return tp if tp is not None and tp.world > 1 else None


def tp_rmsnorm(x: torch.Tensor, scale: torch.Tensor, eps: float, d_full: int, tp: TPGroup) -> torch.Tensor:
    """RMSNorm over the full width of a head-split activation: the per-row sum of
    squares is all-reduced over the tensor-parallel ranks (fp32 statistics).  bf16 CUDA
    rows on the kernel path run ``ops.kernels.tp_norm`` (the result is then bf16)."""
    from .. import ops
    if x.is_cuda and x.dtype == torch.bfloat16 and ops.get_impl() == "cuda" and x.shape[-1] % 256 == 0 \
            and x.shape[-1] <= 8192:
        from ..ops.kernels import tp_norm
        return tp_norm(x, None, scale, eps, d_full, tp)
    xf = x.float()
    ss = tp.all_reduce(xf.square().sum(-1, keepdim=True))
    return xf * torch.rsqrt(ss / d_full + eps) * scale.float()


def tp_norm_gate(x: torch.Tensor, z: torch.Tensor, scale: torch.Tensor, eps: float, d_full: int, tp: TPGroup,
                 zclip: float = float("inf"), oclip: float = float("inf")) -> torch.Tensor:
    """``clamp(rmsnorm_tp(x) * silu(clamp(z, +-zclip)), +-oclip)`` in ``x``'s dtype."""
    import torch.nn.functional as F
    y = tp_rmsnorm(x, scale, eps, d_full, tp).to(x.dtype)
    if zclip != float("inf"):
        z = z.clamp(-zclip, zclip)
    out = y * F.silu(z.to(y.dtype))
    if oclip != float("inf"):
        out = out.clamp(-oclip, oclip)
    return out


def init_tensor_parallel(tp_size: int, device: Optional[torch.device] = None, expert_parallel: bool = False,
                         peer: Optional[bool] = None, max_rows: int = 0, max_width: int = 0) -> TPGroup:
    """Split the job into tensor-parallel groups of ``tp_size`` consecutive ranks and
    install them in the parallel context.  Call before building the model (layers
    size their pieces from the context).  ``expert_parallel``: the routed experts
    are split over the same ranks.  ``peer``: NVLink peer-memory collectives (default:
    on CUDA); ``max_rows`` / ``max_width`` size their buffers (local token rows of a
    micro-batch, widest gathered activation)."""
    from .context import ParallelContext, set_parallel_context
    world, rank = dist.get_world_size(), dist.get_rank()
    if world % tp_size:
        raise ValueError(f"{world} ranks do not split into tensor-parallel groups of {tp_size}")
    groups = [dist.new_group(list(range(i * tp_size, (i + 1) * tp_size))) for i in range(world // tp_size)]
    replicas = None
    if world > tp_size:
        reps = [dist.new_group([j + i * tp_size for i in range(world // tp_size)]) for j in range(tp_size)]
        replicas = reps[rank % tp_size]
    grp = groups[rank // tp_size]
    tp_rank = rank % tp_size
    dev = device or torch.device("cpu")
    if peer is None:
        peer = dev.type == "cuda"
    pt = None
    if peer and dev.type == "cuda" and tp_size > 1:
        from .tp_peer import PeerTP
        pt = PeerTP(tp_size, tp_rank, grp, dev, max_rows, max_width)
    tpg = TPGroup(tp_size, tp_rank, grp, peer=pt)
    ctx = ParallelContext(dp_group=None, dp_world=world, tp_group=grp, tp_world=tp_size, tp_rank=tp_rank,
                          tp=tpg, local_group=replicas)
    if expert_parallel:
        ctx.ep_group, ctx.ep_world, ctx.ep_rank = grp, tp_size, tp_rank
    set_parallel_context(ctx)
    return tpg


@torch.no_grad()
def load_full_state(model: torch.nn.Module, full: dict) -> None:
    """Copy a single-rank state dict into a tensor-parallel model (every split
    parameter takes its piece)."""
    from .context import get_parallel_context
    pc = get_parallel_context()
    for name, p in model.named_parameters():
        t = full[name]
        spec = shard_spec(p)
        if spec is not None and pc.tp_world > 1:
            t = shard_tensor(t, spec[0], spec[1], pc.tp_world, pc.tp_rank)
        elif getattr(p, "_ahb_ep_local", False) and pc.ep_world > 1:
            El = p.shape[0]
            t = t[pc.ep_rank * El:(pc.ep_rank + 1) * El]
        p.copy_(t.to(p.dtype))
