"""Expert parallelism over the GPUs of one node (NVLink peer memory).

The reference replicates every expert on every device (`atomic_ops/moe_gmm.py:84-89`
names EP a follow-up).  Here the routed experts of each MoE layer are split into
``W`` consecutive blocks of ``E / W``; rank ``r`` holds experts
``[r * El, (r + 1) * El)`` and the rows of every token choice travel to the rank of
their expert and back:

forward, per layer
  1. route locally; ``ep_publish`` writes this rank's per-expert counts into every
     peer's count table; peer barrier;
  2. the host reads the ``W x E`` count table and lays out every rank's receive
     buffer: experts in order, 128-row padded segments, sources in rank order
     inside a segment (one small device-to-host copy per layer);
  3. ``ep_dispatch`` stores each token row straight into its expert rank's receive
     buffer (16-byte P2P stores, with the row's (source, assignment) metadata);
     peer barrier;
  4. the local grouped GEMM (tcgen05, SwiGLU/GELU epilogue) runs on the received
     rows; ``ep_return`` stores every output row into the return buffer of its
     source rank at the row of its assignment; peer barrier;
  5. gated combine with the shared expert, locally.
backward: the mirror image -- the row gradients go out with ``ep_dispatch`` (same
positions), the expert backward runs on the receiving rank (weight gradients
stay local: each expert has exactly one owner), and the input-row gradients come
back with ``ep_return``.

Receive buffers are sized for the worst case (every choice of every rank routed to
one rank), so the layout never overflows and the design stays dropless.  The
per-layer host read of the counts rules out CUDA-graph capture of an EP step.
"""
from __future__ import annotations

import os
from typing import List, Optional

import numpy as np
import torch
import torch.distributed as dist

DEFAULT_TIMEOUT_S = float(os.environ.get("AHB_SYMM_TIMEOUT", "120"))


def receive_layout(counts: np.ndarray, rank: int, El: int):
    """Receive-buffer layout from the ``(W, E)`` table of per-source expert counts.

    Rank ``r`` stores its experts ``e = r * El + j`` in order, each in a segment
    padded to a multiple of 128 rows (the grouped GEMM's tile height); inside a
    segment the rows of source ``s`` follow those of sources ``< s``.  Returns, for
    ``rank``: the first destination row of its rows for every expert (``(E,)``, on
    the expert's rank), its own segment offsets (``(El + 1,)``) and sizes (``(El,)``)."""
    cnt = np.asarray(counts, dtype=np.int64)
    W, E = cnt.shape
    segs = cnt.sum(0)
    segp = (segs + 127) // 128 * 128
    off_r = np.zeros((W, El + 1), dtype=np.int64)
    off_r[:, 1:] = np.cumsum(segp.reshape(W, El), axis=1)
    prior = np.cumsum(cnt, axis=0) - cnt
    e = np.arange(E)
    dst_base = off_r[e // El, e % El] + prior[rank]
    return dst_base, off_r[rank], segs.reshape(W, El)[rank]


class EPGroup:
    def __init__(self, world: int, rank: int, n_experts: int, top_k: int, d_model: int, max_tokens: int,
                 device: torch.device, group: Optional[dist.ProcessGroup] = None,
                 timeout_s: float = DEFAULT_TIMEOUT_S):
        from ..ops._ext import ext
        if n_experts % world:
            raise ValueError(f"{n_experts} experts do not split over {world} ranks")
        self.E_ = E = ext()
        self.world, self.rank, self.group = world, rank, group
        self.n_experts, self.k, self.d = n_experts, top_k, d_model
        self.El = n_experts // world
        self.max_tokens = max_tokens
        self.device = device
        self.timeout_s = timeout_s
        self.r_cap = world * max_tokens * top_k + self.El * 128
        sizes = [world * n_experts * 4,              # count table (int32)
                 self.r_cap * d_model * 2,           # receive rows (bf16)
                 self.r_cap * 8,                     # receive metadata (int2)
                 max_tokens * top_k * d_model * 2,   # return rows (bf16)
                 256]                                # barrier pad
        self._own: List[int] = []
        self._opened: List[int] = []
        for n in sizes:
            self._own.append(E.ipc_alloc(n))
        mine = torch.cat([E.ipc_handle(p) for p in self._own]).numpy().tobytes()
        allh: List[Optional[bytes]] = [None] * world
        dist.all_gather_object(allh, mine, group=group)
        ptrs = []
        for r in range(world):
            if r == rank:
                ptrs.append(list(self._own))
                continue
            row = []
            for i in range(len(sizes)):
                p = E.ipc_open(torch.frombuffer(bytearray(allh[r][64 * i:64 * (i + 1)]), dtype=torch.uint8))
                self._opened.append(p)
                row.append(p)
            ptrs.append(row)
        tab = lambda i: torch.tensor([p[i] for p in ptrs], dtype=torch.int64, device=device)  # noqa: E731
        self.count_peers, self.recv_peers, self.meta_peers, self.ret_peers, self.pads = (tab(i) for i in range(5))
        i32 = torch.empty(0, dtype=torch.int32, device=device)
        bf = torch.empty(0, dtype=torch.bfloat16, device=device)
        self.counts = E.ipc_tensor(self._own[0], world * n_experts, i32).view(world, n_experts)
        self.recv = E.ipc_tensor(self._own[1], self.r_cap * d_model, bf).view(self.r_cap, d_model)
        self.meta = E.ipc_tensor(self._own[2], self.r_cap * 2, i32).view(self.r_cap, 2)
        self.ret = E.ipc_tensor(self._own[3], max_tokens * top_k * d_model, bf).view(max_tokens * top_k, d_model)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        self.epoch = 0
        self._host_counts = torch.empty(world, n_experts, dtype=torch.int32, pin_memory=True)
        torch.cuda.synchronize(device)
        dist.barrier(group=group)

    # ------------------------------------------------------------------ plumbing
    def barrier(self) -> None:
        self.epoch += 1
        self.E_.symm_barrier(self.pads, self.rank, self.epoch, self.err, self.timeout_s)

    def check(self) -> None:
        code = int(self.err.item())
        if code:
            raise RuntimeError(f"rank {self.rank}: expert-parallel barrier gave up waiting for rank {code - 100}")

    def layout(self):
        """After the count exchange: this rank's destination bases (E,), and its own
        segment offsets (El + 1,), segment sizes (El,) and row count."""
        self._host_counts.copy_(self.counts)  # synchronising read of the W x E table
        self.check()
        dst_base, off, seg = receive_layout(self._host_counts.numpy(), self.rank, self.El)
        R = int(off[-1])
        assert R <= self.r_cap
        dev = self.device
        mk = lambda a: torch.from_numpy(a.astype(np.int32)).to(dev, non_blocking=False)  # noqa: E731
        return mk(dst_base), mk(off), mk(seg), R

    def close(self) -> None:
        torch.cuda.synchronize(self.device)
        for p in self._opened:
            try:
                self.E_.ipc_close(p)
            except Exception:
                pass
        self._opened = []


class _MoEEP(torch.autograd.Function):
    """Routed experts with expert parallelism (see the module docstring)."""

    @staticmethod
    def forward(ctx, x, top_idx, gate, w1, w2, w3, shared, swiglu, ep):
        E = ep.E_
        bf = torch.bfloat16
        T, k = top_idx.shape
        assert T <= ep.max_tokens, f"{T} tokens > EP capacity {ep.max_tokens}"
        xb = x.to(bf).contiguous()
        eidx, counts, off_local, pos = E.moe_route_local(top_idx, ep.n_experts)
        E.ep_publish(counts, ep.count_peers, ep.rank)
        ep.barrier()
        dst_base, off, seg, R = ep.layout()
        dst_pos = torch.empty(T * k, dtype=torch.int32, device=x.device)
        E.ep_dispatch(xb, True, T, k, eidx, pos, off_local, dst_base, ep.El, ep.recv_peers, ep.meta_peers, ep.rank,
                      dst_pos)
        ep.barrier()
        E.ep_zero_pad(ep.recv, ep.meta, off, seg)
        xs = ep.recv[:R].clone()
        meta = ep.meta[:R].clone()
        w1b, w2b = w1.to(bf).contiguous(), w2.to(bf).contiguous()
        w3b = None if w3 is None else w3.to(bf).contiguous()
        if R > 0:
            a1, a3, h, ys = E.moe_expert_fwd(xs, off, w1b, w2b, w3b, swiglu)
            E.ep_return(ys, meta, R, ep.ret_peers)
        else:  # no token chose this rank's experts
            a1 = a3 = h = xs
        ep.barrier()
        rows = ep.ret[:T * k].clone()
        out = E.moe_combine_rows(rows, gate.float(), None if shared is None else shared.to(bf))
        ctx.save_for_backward(gate, eidx, pos, off_local, dst_base, off, seg, meta, xs, a1, a3, h, rows)
        ctx.w = (w1, w2, w3, w1b, w2b, w3b)
        ctx.ep, ctx.swiglu, ctx.R, ctx.has_shared = ep, swiglu, R, shared is not None
        return out

    @staticmethod
    def backward(ctx, dout):
        from ..ops.kernels import _acc_for, _ret_grad
        gate, eidx, pos, off_local, dst_base, off, seg, meta, xs, a1, a3, h, rows = ctx.saved_tensors
        w1, w2, w3, w1b, w2b, w3b = ctx.w
        ep, R = ctx.ep, ctx.R
        E = ep.E_
        T, k = gate.shape
        drows, dgate = E.moe_combine_rows_bwd(dout.contiguous(), rows, gate)
        E.ep_dispatch(drows, False, T, k, eidx, pos, off_local, dst_base, ep.El, ep.recv_peers, None, ep.rank, None)
        ep.barrier()
        E.ep_zero_pad(ep.recv, None, off, seg)
        a1c, a1d = _acc_for(w1)
        a2c, a2d = _acc_for(w2)
        a3c, a3d = _acc_for(w3) if w3 is not None else (None, False)
        if R > 0:
            dxs = E.moe_expert_bwd(ep.recv[:R], off, xs, a1, a3, h, w1b, w2b, w3b, a1c, a2c, a3c, ctx.swiglu)
            E.ep_return(dxs, meta, R, ep.ret_peers)
        ep.barrier()
        dx = E.moe_sum_rows(ep.ret[:T * k], T, k)
        dshared = dout if ctx.has_shared else None
        return (dx, None, dgate, _ret_grad(w1, a1c, a1d), _ret_grad(w2, a2c, a2d),
                _ret_grad(w3, a3c, a3d) if w3 is not None else None, dshared, None, None)


def moe_forward_ep(x, top_idx, gate, w1, w2, w3, shared, act: str, ep: EPGroup):
    """``x (T, d)``; ``w*`` hold this rank's ``El`` experts."""
    return _MoEEP.apply(x, top_idx, gate, w1, w2, w3, shared, act == "swiglu", ep)


# ------------------------------------------------------------ collective (NCCL / gloo) path
def moe_forward_ep_collective(x, top_idx, gate, w1, w2, w3, act: str, group, world: int, rank: int,
                              n_experts: int):
    """Expert parallelism with ``torch.distributed`` all-to-all (NCCL on GPUs, gloo on the
    CPU): the baseline of the peer-memory path above and the path without peer buffers.

    Every token choice ``(t, j)`` travels to the rank of expert ``top_idx[t, j]`` (rows
    grouped by destination, then by expert), the experts run there on the rows grouped by
    expert, and the outputs travel back in the order they came; the combine
    ``sum_j gate[t, j] * y[t, j]`` happens on the token's rank.  Differentiable (the
    all-to-all's backward is the reverse all-to-all).  Returns the fp32 routed output
    ``(T, d)`` before the shared expert and the final sanitize."""
    import torch.distributed.nn.functional as dfn
    from .. import ops
    from ..ops import reference as R
    T, k = top_idx.shape
    El = n_experts // world
    eidx = top_idx.reshape(-1)                                   # assignment a = t * k + j
    order = torch.argsort(eidx, stable=True)                     # by expert = by destination, then expert
    counts = torch.bincount(eidx, minlength=n_experts)           # (E,) rows this rank sends per expert
    allc = [torch.zeros_like(counts) for _ in range(world)]
    dist.all_gather(allc, counts, group=group)
    table = torch.stack(allc).cpu()                              # (W, E): rows from source s for expert e
    send = table[rank].view(world, El).sum(1).tolist()           # rows to each destination rank
    recv = table[:, rank * El:(rank + 1) * El].sum(1).tolist()   # rows from each source rank
    rows = x[order // k]
    got = dfn.all_to_all_single(rows.new_empty((sum(recv), x.shape[1])), rows, recv, send, group=group)
    # received rows: source-major, expert-major inside a source -> regroup by local expert
    src_e = torch.cat([torch.arange(El).repeat_interleave(table[s, rank * El:(rank + 1) * El])
                       for s in range(world)]) if sum(recv) else torch.zeros(0, dtype=torch.long)
    regroup = torch.argsort(src_e.to(x.device), stable=True)
    sizes = table[:, rank * El:(rank + 1) * El].sum(0).tolist()
    ys = ops.grouped_ffn(got[regroup], torch.tensor(sizes), w1, w2, w3, act, group_sizes_cpu=sizes)
    ys = R.sanitize(ys.float(), 1e3)
    back = torch.empty_like(ys)
    back = back.index_copy(0, regroup, ys)                       # undo the regrouping (differentiable)
    out_rows = dfn.all_to_all_single(back.new_empty((T * k, back.shape[1])), back, send, recv, group=group)
    y = torch.empty_like(out_rows).index_copy(0, order, out_rows)  # assignment order t * k + j
    return (y.view(T, k, -1) * gate.float().unsqueeze(-1)).sum(1)


def init_expert_parallel(ep_size: int):
    """Expert-parallel groups of ``ep_size`` consecutive ranks; with ``ep_size < world`` the
    ``world / ep_size`` groups are data-parallel replicas of one another: every rank reads
    its own tokens, the routed experts are split within a group, and the gradients of a
    block of experts are summed over the ranks that hold the same block (``local_group``)
    before the step.  Installs the layout in the parallel context and returns it."""
    from .context import ParallelContext, set_parallel_context
    world, rank = dist.get_world_size(), dist.get_rank()
    if world % ep_size:
        raise ValueError(f"{world} ranks do not split into expert-parallel groups of {ep_size}")
    ctx = ParallelContext(dp_world=world, ep_world=ep_size, ep_rank=rank % ep_size)
    if ep_size < world:
        reps = world // ep_size
        for i in range(reps):  # every rank creates every group, in the same order
            g = dist.new_group(list(range(i * ep_size, (i + 1) * ep_size)))
            if i == rank // ep_size:
                ctx.ep_group = g
        for j in range(ep_size):
            g = dist.new_group([j + i * ep_size for i in range(reps)])
            if j == rank % ep_size:
                ctx.local_group = g
    set_parallel_context(ctx)
    return ctx
