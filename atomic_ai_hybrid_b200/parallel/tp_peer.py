"""Tensor-parallel collectives over NVLink peer memory (one node, one process per GPU).

Every rank allocates, with ``cudaMalloc``, and shares through CUDA IPC handles:

* two send buffers (``max_rows x max_width`` bf16): a rank publishes its token rows
  there for the all-gather;
* two receive buffers (``W`` slots of ``max_rows x max_width`` bf16): slot ``s`` holds
  the partial sums that rank ``s`` owes this rank in a reduce-scatter;
* a barrier pad (``parallel.symm`` protocol: bounded waits, error word).

Calls alternate between the two buffers of each kind and every call runs one peer
barrier between its writes and its reads.  A buffer is written again two calls
later, after the barrier of the call in between, which every rank reaches only when
it has finished reading the buffer - so no call overwrites rows a peer still reads.

All-gather (``all_gather_rows``): publish the local rows (one local copy), barrier,
then the GPU's copy engines pull the peers' rows over NVLink (``cudaMemcpyAsync`` on a
side stream, one event per source) while the compute stream consumes the rows that
are present - its own first - so the transfer of rank ``s``'s rows overlaps the
projections of the rows before them.

Reduce-scatter (``reduce_scatter_rows``): the partial rows owed to every peer are
pushed by the copy engines into that peer's receive slot (the producer of the rows
for the next peer runs meanwhile), barrier, then one kernel sums the slots.

Row-parallel projection (``linear_scatter``): one tcgen05 GEMM computes every
rank's partial rows and its epilogue stores each tile straight into the owner's
receive slot (16-byte peer stores; no copy of the partial product exists), then the
barrier and the slot sum.  The tiles are visited from the next rank's rows on, so
the ranks write to different peers at any time.

No TMA load touches peer memory (the GEMM's operands are local), no library kernel
gets a peer's buffer as an operand, and nothing uses multicast.
"""
from __future__ import annotations

import os
from typing import Callable, List, Optional, Tuple

import torch
import torch.distributed as dist

DEFAULT_TIMEOUT_S = float(os.environ.get("AHB_SYMM_TIMEOUT", "120"))


class PeerTP:
    def __init__(self, world: int, rank: int, group: Optional[dist.ProcessGroup], device: torch.device,
                 max_rows: int, max_width: int, timeout_s: float = DEFAULT_TIMEOUT_S):
        from ..ops._ext import ext
        if max_rows <= 0 or max_width <= 0:
            raise ValueError("PeerTP needs max_rows and max_width (local token rows, widest row)")
        if world > 8:
            raise ValueError("peer tensor parallelism supports at most 8 ranks")
        self.E = E = ext()
        self.world, self.rank, self.group = world, rank, group
        self.device = device
        self.max_rows, self.max_width = max_rows, max_width
        self.timeout_s = float(timeout_s)
        self.slot = max_rows * max_width  # elements of one slot / send buffer
        sizes = [self.slot * 2, self.slot * 2, world * self.slot * 2, world * self.slot * 2, 256]
        self._own: List[int] = []
        self._opened: List[int] = []
        try:
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
                    h = torch.frombuffer(bytearray(allh[r][64 * i:64 * (i + 1)]), dtype=torch.uint8)
                    p = E.ipc_open(h)
                    self._opened.append(p)
                    row.append(p)
                ptrs.append(row)
        except Exception:
            self._release(free_own=True)
            raise
        self.send = [[ptrs[r][b] for r in range(world)] for b in range(2)]      # send[b][r]
        self.recv = [[ptrs[r][2 + b] for r in range(world)] for b in range(2)]  # recv[b][r]
        self.pads = torch.tensor([p[4] for p in ptrs], dtype=torch.int64, device=device)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        self._err_host = torch.zeros(1, dtype=torch.int32, pin_memory=True)
        self._err_ev = torch.cuda.Event()
        self._err_pending = False
        self.epoch = 0
        self._n_send = 0
        self._n_recv = 0
        self.copy_stream = torch.cuda.Stream(device=device)
        self._offs = {}
        self.closed = False
        torch.cuda.synchronize(device)
        dist.barrier(group=group)

    # ------------------------------------------------------------ checks
    def usable(self, x: torch.Tensor) -> bool:
        if self.closed or not x.is_cuda or x.dtype != torch.bfloat16:
            return False
        w = x.shape[-1]
        rows = x.numel() // w
        return w % 8 == 0 and w <= self.max_width and rows <= self.world * self.max_rows

    def poll(self) -> None:
        if self._err_pending and self._err_ev.query():
            self._err_pending = False
            code = int(self._err_host[0])
            if code:
                raise RuntimeError(f"rank {self.rank}: tensor-parallel peer barrier gave up waiting for rank "
                                   f"{code - 100} after {self.timeout_s:.0f} s")

    def barrier(self) -> None:
        self.epoch += 1
        self.E.symm_barrier(self.pads, self.rank, self.epoch, self.err, self.timeout_s)
        if not self._err_pending:
            self._err_host.copy_(self.err, non_blocking=True)
            self._err_ev.record()
            self._err_pending = True

    # ------------------------------------------------------------ all-gather
    def all_gather_rows(self, x: torch.Tensor,
                        consume: Optional[Callable[[int, slice, torch.Tensor], None]] = None) -> torch.Tensor:
        """``(n, w)`` local rows -> ``(W n, w)`` rows of all ranks in rank order.
        ``consume(s, rows, full)`` runs on the compute stream as soon as the rows of
        rank ``s`` are present (own rows first)."""
        self.poll()
        x = x.contiguous()
        n, w = x.shape
        if n * w > self.slot:
            raise ValueError(f"all_gather_rows: {n} x {w} rows exceed the peer buffers")
        nbytes = n * w * 2
        b = self._n_send % 2
        self._n_send += 1
        cur = torch.cuda.current_stream(self.device)
        E = self.E
        E.memcpy_async(self.send[b][self.rank], x.data_ptr(), nbytes, cur.cuda_stream)
        self.barrier()
        full = torch.empty((self.world * n, w), dtype=x.dtype, device=x.device)
        ready = torch.cuda.Event()
        ready.record(cur)
        cs = self.copy_stream
        cs.wait_event(ready)
        order = [(self.rank + i) % self.world for i in range(1, self.world)]
        evs = {}
        for s in order:
            E.memcpy_async(full[s * n:(s + 1) * n].data_ptr(), self.send[b][s], nbytes, cs.cuda_stream)
            ev = torch.cuda.Event()
            ev.record(cs)
            evs[s] = ev
        full[self.rank * n:(self.rank + 1) * n].copy_(x)
        if consume is not None:
            consume(self.rank, slice(self.rank * n, (self.rank + 1) * n), full)
        for s in order:
            cur.wait_event(evs[s])
            if consume is not None:
                consume(s, slice(s * n, (s + 1) * n), full)
        return full

    # ------------------------------------------------------------ reduce-scatter
    def reduce_scatter_rows(self, y: Optional[torch.Tensor], n: Optional[int] = None, w: Optional[int] = None,
                            produce: Optional[Callable[[int, slice], torch.Tensor]] = None) -> torch.Tensor:
        """Partial ``(W n, w)`` rows -> this rank's ``(n, w)`` sums over the ranks.
        With ``produce(s, rows)`` the partial rows owed to rank ``s`` are computed on
        the compute stream just before they are pushed (next peer first, own last)."""
        self.poll()
        if y is not None:
            y = y.contiguous()
            n, w = y.shape[0] // self.world, y.shape[1]
        if n * w > self.slot:
            raise ValueError(f"reduce_scatter_rows: {n} x {w} rows exceed the peer buffers")
        nbytes = n * w * 2
        b = self._n_recv % 2
        self._n_recv += 1
        cur = torch.cuda.current_stream(self.device)
        cs = self.copy_stream
        E = self.E
        keep = []
        for i in range(1, self.world + 1):
            s = (self.rank + i) % self.world
            part = produce(s, slice(s * n, (s + 1) * n)) if produce is not None else y[s * n:(s + 1) * n]
            part = part.contiguous()
            dst = self.recv[b][s] + self.rank * self.slot * 2
            if s == self.rank:
                E.memcpy_async(dst, part.data_ptr(), nbytes, cur.cuda_stream)
            else:
                ev = torch.cuda.Event()
                ev.record(cur)
                cs.wait_event(ev)
                E.memcpy_async(dst, part.data_ptr(), nbytes, cs.cuda_stream)
                part.record_stream(cs)
            keep.append(part)
        done = torch.cuda.Event()
        done.record(cs)
        cur.wait_event(done)
        self.barrier()
        out = torch.empty((n, w), dtype=torch.bfloat16, device=self.device)
        E.sum_slots(self.recv[b][self.rank], self.world, self.slot, out)
        return out

    # ------------------------------------------------------------ fused row-parallel projection
    def _grp_off(self, n: int) -> torch.Tensor:
        t = self._offs.get(n)
        if t is None:
            t = torch.arange(self.world + 1, dtype=torch.int32, device=self.device) * n
            self._offs[n] = t
        return t

    def gemm_rs(self, a: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        """``(W n, K) @ (K, N)`` summed over the ranks, this rank's ``(n, N)`` rows;
        the partial tiles travel from the GEMM epilogue into the owners' slots."""
        self.poll()
        a = a.contiguous()
        N = w.shape[1]
        n = a.shape[0] // self.world
        if n * N > self.slot:
            raise ValueError("gemm_rs: output rows exceed the peer buffers")
        b = self._n_recv % 2
        self._n_recv += 1
        outs = [self.recv[b][g] + self.rank * self.slot * 2 for g in range(self.world)]
        m_rot = ((self.rank + 1) % self.world) * (n // 128)
        self.E.tp_gemm_rs(a, w.contiguous(), self._grp_off(n), outs, m_rot)
        self.barrier()
        out = torch.empty((n, N), dtype=torch.bfloat16, device=self.device)
        self.E.sum_slots(self.recv[b][self.rank], self.world, self.slot, out)
        return out

    def gemm_rs_ok(self, a: torch.Tensor, w: torch.Tensor) -> bool:
        n = a.shape[0] // self.world
        return (a.shape[0] % self.world == 0 and n % 128 == 0 and a.shape[1] % 64 == 0 and w.shape[1] % 32 == 0
                and w.dtype == torch.bfloat16 and n * w.shape[1] <= self.slot)

    # ------------------------------------------------------------ layer edges (autograd)
    def gather_linear(self, x: torch.Tensor, pairs, batch_shape: Tuple[int, int]):
        ws = [w for w, _ in pairs]
        bs = [b for _, b in pairs]
        outs = _PeerGatherLinear.apply(x.reshape(-1, x.shape[-1]), self, len(pairs), *ws, *bs)
        return [o.view(*batch_shape, o.shape[-1]) for o in outs]

    def linear_scatter(self, o: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        return _PeerLinearScatter.apply(o.reshape(-1, o.shape[-1]), self, w).unsqueeze(0)

    # ------------------------------------------------------------ teardown
    def _release(self, free_own: bool) -> None:
        for p in self._opened:
            try:
                self.E.ipc_close(p)
            except Exception:
                pass
        self._opened = []
        if free_own:
            for p in self._own:
                try:
                    self.E.ipc_free(p)
                except Exception:
                    pass
            self._own = []

    def close(self) -> None:
        if self.closed:
            return
        self.closed = True
        torch.cuda.synchronize(self.device)
        self._release(free_own=False)


def _bf16(w: torch.Tensor) -> torch.Tensor:
    return w if w.dtype == torch.bfloat16 else w.to(torch.bfloat16)


class _PeerGatherLinear(torch.autograd.Function):
    """``[gather(x) W_i + b_i]``: the projections of each rank's rows start as soon as
    those rows arrive.  Backward: the partial input gradients owed to each rank are
    computed just before they are pushed, the weight gradients use the gathered rows
    kept from the forward."""

    @staticmethod
    def forward(ctx, x, peer, n, *wb):
        ws, bs = wb[:n], wb[n:]
        wcs = [_bf16(w) for w in ws]
        T = x.shape[0] * peer.world
        outs = [torch.empty((T, w.shape[1]), dtype=torch.bfloat16, device=x.device) for w in ws]

        def consume(s, rows, full):
            xs = full[rows]
            for o, wc, b in zip(outs, wcs, bs):
                if b is not None:
                    torch.addmm(b.to(torch.bfloat16), xs, wc, out=o[rows])
                else:
                    torch.mm(xs, wc, out=o[rows])

        full = peer.all_gather_rows(x.to(torch.bfloat16), consume)
        ctx.save_for_backward(full, *ws)
        ctx.peer, ctx.n, ctx.has_b = peer, n, [b is not None for b in bs]
        ctx.bs = list(bs)
        return tuple(outs)

    @staticmethod
    def backward(ctx, *dys):
        from ..ops.kernels import _wgrad_acc, bias_grad
        full, *ws = ctx.saved_tensors
        peer = ctx.peer
        wcs = [_bf16(w) for w in ws]
        dys = [None if d is None else d.reshape(-1, d.shape[-1]).to(torch.bfloat16) for d in dys]
        n = full.shape[0] // peer.world
        d = full.shape[1]
        dx = None
        if ctx.needs_input_grad[0]:
            def produce(s, rows):
                acc = None
                for dy, wc in zip(dys, wcs):
                    if dy is None:
                        continue
                    if acc is None:
                        acc = torch.mm(dy[rows], wc.t())
                    else:
                        torch.addmm(acc, dy[rows], wc.t(), out=acc)
                return acc if acc is not None else torch.zeros((n, d), dtype=torch.bfloat16, device=full.device)
            dx = peer.reduce_scatter_rows(None, n, d, produce)
        dws, dbs = [], []
        for w, dy, hb in zip(ws, dys, ctx.has_b):
            if dy is None:
                dws.append(None)
                dbs.append(None)
                continue
            acc = getattr(w, "_ahb_grad_acc", None)
            if acc is not None and w.dtype != torch.float32:
                _wgrad_acc(acc.view(w.shape), full, dy)
                dws.append(None)
            else:
                dws.append((full.t() @ dy).to(w.dtype))
            dbs.append(bias_grad(ctx.bs[len(dbs)], dy) if hb else None)
        return (dx, None, None, *dws, *dbs)


class _PeerLinearScatter(torch.autograd.Function):
    """Row-parallel ``o W`` reduce-scattered to token rows: the tcgen05 GEMM with the
    peer-store epilogue when the shapes allow, else cuBLAS + the copy-engine push.
    Backward: the output-row gradients are all-gathered and ``dO`` for each rank's
    rows is computed as they arrive."""

    @staticmethod
    def forward(ctx, o, peer, w):
        ob = o.to(torch.bfloat16).contiguous()
        wc = _bf16(w).contiguous()
        if peer.gemm_rs_ok(ob, wc):
            y = peer.gemm_rs(ob, wc)
        else:
            y = peer.reduce_scatter_rows(ob @ wc)
        ctx.save_for_backward(ob, w)
        ctx.peer = peer
        return y

    @staticmethod
    def backward(ctx, dy):
        from ..ops.kernels import _wgrad_acc
        ob, w = ctx.saved_tensors
        peer = ctx.peer
        wc = _bf16(w)
        do = torch.empty_like(ob) if ctx.needs_input_grad[0] else None

        def consume(s, rows, full):
            if do is not None:
                torch.mm(full[rows], wc.t(), out=do[rows])

        dyf = peer.all_gather_rows(dy.contiguous().to(torch.bfloat16), consume)
        acc = getattr(w, "_ahb_grad_acc", None)
        if acc is not None and w.dtype != torch.float32:
            _wgrad_acc(acc.view(w.shape), ob, dyf)
            dw = None
        else:
            dw = (ob.t() @ dyf).to(w.dtype)
        return do, None, dw
