"""Train step: gradient accumulation over micro-batches, then the sharded apply.

One ``Trainer`` per process (one process per GPU).  ``micro_step`` runs the
forward/backward of one micro-batch and accumulates fp32 gradients in the flat
store (reference ``distributed_train_step_micro``, `train_setup.py:477-488`);
``apply`` reduces gradients across the data-parallel group onto their owner
ranks, runs the hybrid optimizer on the owned shard and gathers the updated
weights back to every rank (reference ``distributed_apply_step``,
`train_setup.py:490-550`).  The assignment fractions used by the expert-bias
hook are averaged over the micro-steps of the step and over ranks.

With ``cuda_graph=True`` the whole micro-step (forward, loss, backward and the
gradient accumulation into the store) is captured once as a CUDA graph and
replayed for every micro-batch of the same shape: one launch per micro-step
instead of thousands.  The graph is built at the start of a step (its warm-up
iterations are discarded by zeroing the gradients before the real micro-steps).
"""
from __future__ import annotations

import os
from typing import Dict, List, Optional

import torch
import torch.distributed as dist

from ..optim import FlatParamStore, HybridOptimizer, grad_scale_of, label_adamw_only, label_of
from ..optim.store import is_ep_local
from .loss import compute_loss
from ..utils.diag import DIAG
from ..utils.nvtx import nvtx_range


class Trainer:
    def __init__(self, model, total_steps: int = 1000, optimizer: str = "hybrid",
                 compute_dtype: torch.dtype = torch.bfloat16, device=None,
                 group: Optional[dist.ProcessGroup] = None, comm: str = "auto",
                 ce_chunk_size: int = 2048, collinearity_coef: Optional[float] = None,
                 skip_nonfinite: bool = False, cuda_graph: bool = False, ep_max_tokens: int = 0,
                 offload_local_moments: bool = False, expert_grad_bf16: bool = False):
        self.model = model
        self.cfg = model.cfg
        self.group = group
        dist_on = dist.is_available() and dist.is_initialized()
        self.world = dist.get_world_size(group) if dist_on else 1
        self.rank = dist.get_rank(group) if dist_on else 0
        label_fn = label_of if optimizer == "hybrid" else label_adamw_only
        ep_params = any(is_ep_local(n, p) for n, p in model.named_parameters())
        self.store = FlatParamStore(model, label_fn, grad_scale_of, self.world, self.rank,
                                    compute_dtype=compute_dtype, device=device,
                                    param_filter=(lambda n, p: not is_ep_local(n, p)) if ep_params else None)
        # rank-local parameters (expert-parallel experts, tensor-parallel pieces): a local
        # store (no reduce-scatter / all-gather) stepped with the main one; when the same
        # piece lives on several ranks (data-parallel replicas of a tensor-parallel
        # group) its gradients are summed over ``local_group`` before the step
        from ..parallel.context import get_parallel_context
        self.local_group = get_parallel_context().local_group
        self.ep_store = None
        # ``expert_grad_bf16``: the expert-parallel experts get a local store of their own with
        # bf16 gradient accumulators (the MoE weight-gradient GEMMs add into them, rounding once
        # per micro-step); the tensor-parallel pieces keep fp32 ones in ``ep_store``
        self.xp_store = None
        if ep_params:
            experts = (lambda n, p: bool(getattr(p, "_ahb_ep_local", False))) if expert_grad_bf16 else None
            if experts is not None and any(experts(n, p) for n, p in model.named_parameters()):
                self.xp_store = FlatParamStore(model, label_fn, grad_scale_of, 1, 0, compute_dtype=compute_dtype,
                                               device=device, param_filter=experts, grad_dtype=torch.bfloat16)
                rest = lambda n, p: is_ep_local(n, p) and not experts(n, p)  # noqa: E731
            else:
                rest = is_ep_local
            if any(rest(n, p) for n, p in model.named_parameters()):
                self.ep_store = FlatParamStore(model, label_fn, grad_scale_of, 1, 0, compute_dtype=compute_dtype,
                                               device=device, param_filter=rest)
        self.comm = None
        if self.world > 1:
            from ..parallel.context import ParallelContext, set_parallel_context
            pc = get_parallel_context()
            if pc.dp_world != self.world and pc.tp is None and pc.ep_world <= 1:
                set_parallel_context(ParallelContext(dp_group=group, dp_world=self.world))
            from ..parallel.fsdp import make_shard_comm
            self.comm = make_shard_comm(self.store, group, comm)
        self.opt = HybridOptimizer(self.store, total_steps, reduce_fn=self._allreduce_sum,
                                   skip_nonfinite=skip_nonfinite)
        self.ep_opt = self.xp_opt = None
        for name in ("ep", "xp"):
            st = getattr(self, f"{name}_store")
            if st is None:
                continue
            # ``offload_local_moments``: the rank-local parameters' AdamW moments in host memory
            o = HybridOptimizer(st, total_steps, offload_moments=offload_local_moments)
            o.schedule = self.opt.schedule  # one learning-rate schedule for every store
            if self.local_group is not None:
                # every replica adds the same statistics to the cross-rank sum
                o.norm_share = 1.0 / dist.get_world_size(self.local_group)
            self.opt.partners.append(o)
            setattr(self, f"{name}_opt", o)
        if self.local_stores():
            pc = get_parallel_context()
            if pc.tp is not None and pc.tp.world > 1:
                # the head-split layers run eager (per-call peer barriers carry host epochs)
                cuda_graph = False
            if pc.ep_world > 1:
                # peer buffers on CUDA (AHB_EP_COMM=nccl keeps the all-to-all baseline); on the
                # CPU the MoE uses the torch.distributed all-to-all path
                peer = self.store.device.type == "cuda" and os.environ.get("AHB_EP_COMM", "peer") != "nccl"
                if pc.ep is None and peer:
                    if ep_max_tokens <= 0:
                        raise ValueError("expert parallelism needs ep_max_tokens (tokens per micro-batch)")
                    from ..parallel.ep import EPGroup
                    pc.ep = EPGroup(pc.ep_world, pc.ep_rank, self.cfg.e_routed, self.cfg.top_k, self.cfg.d_model,
                                    ep_max_tokens, self.store.device, group=pc.ep_group)
                # the per-layer host read of the routing counts cannot be captured
                cuda_graph = False
        # peer-memory comm + fused optimizer kernels: reduce-scatter and all-gather
        # happen inside the optimizer's prepare / apply kernels
        self.fused_comm = bool(self.comm is not None and getattr(self.comm, "fused", False)
                               and self.opt.uses_kernels())
        if self.fused_comm:
            self.opt.peers = (self.comm.grad_peers, self.comm.compute_peers)
        self.ce_chunk_size = ce_chunk_size
        self.collinearity_coef = collinearity_coef
        self.global_step = 0
        dev = self.store.device
        n_moe = sum(1 for n, _ in model.named_parameters() if n.endswith("expert_bias"))
        self._frac_sum = torch.zeros(max(n_moe, 1), self.cfg.e_routed, device=dev)
        self._loss_sum = torch.zeros((), device=dev)
        self._n_micro = 0
        self.cuda_graph = cuda_graph and dev.type == "cuda"
        self.phase_events = None  # dict name -> [cuda.Event] when a caller times the step phases
        if dev.type == "cuda":
            # the model's construction-time parameter tensors were replaced by views of the
            # flat store: hand their cached blocks back so that libraries allocating outside
            # PyTorch's cache (cuBLAS handles and workspaces) find memory
            torch.cuda.empty_cache()
        self._graph = None
        self._graph_key = None
        self.graph_kernel_launches = 0
        self.last_info: Optional[Dict] = None

    def _allreduce_sum(self, t: torch.Tensor) -> torch.Tensor:
        if self.world > 1:
            dist.all_reduce(t, group=self.group)
        return t

    # ------------------------------------------------------------ micro-step
    def _micro_body(self, batch: Dict[str, torch.Tensor]):
        self.model.train()
        with nvtx_range("forward"):
            loss, info = compute_loss(self.model, batch, deterministic=False, ce_chunk_size=self.ce_chunk_size,
                                      collinearity_coef=self.collinearity_coef)
        with nvtx_range("backward"):
            loss.backward()
        if info.get("assignment_frac") is not None:
            self._frac_sum += info["assignment_frac"]
        self._loss_sum += loss.detach()
        return loss.detach(), info

    def micro_step(self, batch: Dict[str, torch.Tensor]):
        if self.cuda_graph and self._graph is not None and self._graph_key == self._key(batch):
            self._s_ids.copy_(batch["input_ids"])
            self._s_lab.copy_(batch["labels"])
            self._graph.replay()
            self._n_micro += 1
            self.last_info = self._s_info
            return self._s_loss, self._s_info
        out = self._micro_body(batch)
        self._n_micro += 1
        self.last_info = out[1]  # the step's statistics, read by the loop on logging steps
        return out

    @staticmethod
    def _key(batch):
        return tuple(batch["input_ids"].shape), batch["input_ids"].dtype

    def build_graph(self, batch: Dict[str, torch.Tensor], warmup: int = 2) -> None:
        """Capture one micro-step for this batch shape.  Leaves gradients zeroed."""
        from ..utils.counters import launch_counter
        self._s_ids = batch["input_ids"].clone()
        self._s_lab = batch["labels"].clone()
        sb = {"input_ids": self._s_ids, "labels": self._s_lab}
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(warmup):
                self._micro_body(sb)
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        before = launch_counter.count
        was_on = launch_counter.on
        launch_counter.enable()
        with torch.cuda.graph(g):
            self._s_loss, self._s_info = self._micro_body(sb)
        if not was_on:
            launch_counter.disable()
        self.graph_kernel_launches = launch_counter.count - before
        launch_counter.count = before
        torch.cuda.synchronize()
        self._graph = g
        self._graph_key = self._key(batch)
        self.reset_accumulators()

    def local_stores(self):
        """The rank-local stores (tensor-parallel pieces / experts; experts separately with
        bf16 gradients under ``expert_grad_bf16``)."""
        return [st for st in (self.ep_store, self.xp_store) if st is not None]

    def reset_accumulators(self) -> None:
        self.store.zero_grad()
        for st in self.local_stores():
            st.zero_grad()
        self._frac_sum.zero_()
        self._loss_sum.zero_()
        self._n_micro = 0

    # ------------------------------------------------------------ apply
    def _mark(self, name: str) -> None:
        """Record a CUDA event at a phase boundary when the caller asked for phase timing
        (``self.phase_events`` is a dict name -> list of events; off by default)."""
        if self.phase_events is not None:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            self.phase_events.setdefault(name, []).append(e)

    def apply(self, n_accum: Optional[int] = None) -> Dict[str, torch.Tensor]:
        self._mark("apply")
        n = n_accum if n_accum is not None else max(self._n_micro, 1)
        frac = None
        if self._n_micro > 0:
            frac = self._frac_sum / self._n_micro
            if self.world > 1:
                dist.all_reduce(frac, group=self.group)
                frac = frac / self.world
        if self.local_group is not None:
            for st in self.local_stores():
                dist.all_reduce(st.grad, group=self.local_group)
        if self.fused_comm:
            self.comm.begin_step()
        elif self.comm is not None:
            self.comm.reduce_scatter_grads()
        self._mark("optimizer")
        # every rank's loss is the mean over its own tokens, and the reduction sums the
        # ranks: dividing by n_accum * world gives the gradient of the global-batch mean
        with nvtx_range("optimizer"):
            out = self.opt.step(n * self.world, frac)
        self._mark("end_barrier")
        if self.fused_comm:
            self.comm.end_step()
        elif self.comm is not None:
            self.comm.all_gather_params()
        self._mark("done")
        out["loss"] = self._loss_sum / max(self._n_micro, 1)
        self.reset_accumulators()
        # step diagnostics: the previous step's events print now ([FWD-DIAG], [RESID-DIAG], ...)
        DIAG.end_step(self.global_step)
        self.global_step += 1
        return out

    def train_step(self, micro_batches: List[Dict[str, torch.Tensor]]):
        if self.cuda_graph and (self._graph is None or self._graph_key != self._key(micro_batches[0])):
            self.build_graph(micro_batches[0])
        self._mark("micro")
        for b in micro_batches:
            self.micro_step(b)
        return self.apply(len(micro_batches))

    def close(self) -> None:
        """Release the captured CUDA graph.  A graph that contains NCCL collectives
        (the data-parallel MoE statistics) must be released before the process
        group is destroyed, or the teardown waits on it forever."""
        if self._graph is not None:
            torch.cuda.synchronize()
            self._graph.reset()
            self._graph = None
            self._graph_key = None
            self._s_loss = self._s_info = None
            torch.cuda.synchronize()
        if self.comm is not None and hasattr(self.comm, "close"):
            self.comm.close()
        if self.local_stores():
            from ..parallel.context import get_parallel_context
            pc = get_parallel_context()
            if pc.ep is not None:
                pc.ep.close()
            if pc.tp is not None:
                pc.tp.close()

    @torch.no_grad()
    def eval_loss(self, batch: Dict[str, torch.Tensor]) -> torch.Tensor:
        self.model.eval()
        loss, _ = compute_loss(self.model, batch, deterministic=True, ce_chunk_size=self.ce_chunk_size)
        self.model.train()
        return loss
