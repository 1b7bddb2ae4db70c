"""Pipeline parallelism for the interleaved stack (1F1B or GPipe schedule over NCCL / gloo p2p).

The reference has no pipeline parallelism (GSPMD FSDP + DP on a 1-D mesh,
`train_setup.py:361-365`); here it is an additional layout whose stage-to-stage sends and
receives run on NCCL (or gloo) point-to-point.  Stage ``s`` of ``S`` runs a
contiguous block of the layers; the first stage also embeds the tokens and the last one
applies the final norm and the tied LM head, for which it holds a copy of the embedding
table whose gradient is summed with the first stage's before every optimizer step (both
copies then take the same update).

One optimizer step (``micro_step`` per micro-batch, then ``apply``; ``train_step`` does
both) runs one of two schedules over the step's micro-batches:

* ``"1f1b"`` (default): stage ``s`` runs ``S - s - 1`` warm-up forwards, then alternates
  one forward and one backward, then drains the remaining backwards, so at most ``S - s``
  micro-batches hold activations at once.  Where a stage sends an activation forward and
  receives a gradient back (or the reverse) in the same slot, the two transfers go out as
  one batched pair (``batch_isend_irecv``): the two neighbours then issue their transfers
  over the link in the same order, and neither blocks the other.
* ``"gpipe"``: every micro-batch forward, then every micro-batch backward.

Each stage adds the MoE auxiliary terms of its own layers to its backward seed, so the
gradient of every parameter is that of the single-rank loss.  The global gradient norm, the
clip coefficient and the non-finite flags are reduced over every rank.  Parameters keep
their global names, so checkpoints are interchangeable with the other layouts.

With ``data_parallel = D > 1`` the job is a ``D x S`` mesh (rank ``d S + s`` is stage ``s``
of replica ``d``): each replica reads its own share of the batch, each stage's flat store is
sharded over the ``D`` ranks that hold that stage (gradient reduce-scatter and parameter
all-gather over that group), and the tied embedding is summed between the first and last
stage of each replica before the data-parallel reduction.
"""
from __future__ import annotations

from typing import Dict, List, Optional

import torch
import torch.distributed as dist
import torch.nn as nn


def stage_layers(num_layers: int, stages: int, stage: int) -> range:
    """Contiguous, balanced layer ranges: the first ``num_layers % stages`` stages take one more."""
    base, extra = divmod(num_layers, stages)
    lo = stage * base + min(stage, extra)
    return range(lo, lo + base + (1 if stage < extra else 0))


class PipelineStage(nn.Module):
    """The modules of one stage, registered under the model's own attribute names."""

    def __init__(self, model: nn.Module, stages: int, stage: int):
        super().__init__()
        if model.cfg.arch != "interleaved":
            raise ValueError("pipeline parallelism splits the interleaved layout")
        self.cfg = model.cfg
        self.compute_dtype = model.compute_dtype
        self.stages, self.stage = stages, stage
        self.first, self.last = stage == 0, stage == stages - 1
        self.layer_ids = list(stage_layers(model.cfg.num_layers, stages, stage))
        for i in self.layer_ids:
            setattr(self, f"layer_{i}", getattr(model, f"layer_{i}"))
        if self.first or (self.last and model.cfg.tie_embeddings):
            self.embed = model.embed
        if self.last:
            self.final_norm = model.final_norm
            if not model.cfg.tie_embeddings:
                self.lm_head = model.lm_head
        self._model = [model]  # for rope / lm_weight helpers (not a registered submodule)

    def run(self, x: torch.Tensor, seq_len: int, stats: List[Dict]) -> torch.Tensor:
        m = self._model[0]
        cos, sin = m.rope(seq_len, x.device) if m.has_mla() else (None, None)
        for i in self.layer_ids:
            x = getattr(self, f"layer_{i}")(x, cos, sin, stats)
        return x


def pipeline_groups(stages: int, data_parallel: int = 1):
    """Process groups of a ``data_parallel x stages`` mesh (rank ``d * stages + s``).

    Every rank creates every group in the same order (``new_group`` is collective).
    Returns ``(pp_group, pp_ranks, dp_group, tied_group)`` for the calling rank; a group
    that would span the whole job is ``None`` (the default group)."""
    world, rank = dist.get_world_size(), dist.get_rank()
    if stages * data_parallel != world:
        raise ValueError(f"pipeline mesh {data_parallel} x {stages} does not cover {world} ranks")
    d, s = divmod(rank, stages)
    pp_group = dp_group = tied_group = None
    pp_ranks = list(range(d * stages, (d + 1) * stages))
    if data_parallel > 1:
        for dd in range(data_parallel):
            g = dist.new_group(list(range(dd * stages, (dd + 1) * stages)))
            if dd == d:
                pp_group = g
        if stages > 1:
            for ss in range(stages):
                g = dist.new_group([dd * stages + ss for dd in range(data_parallel)])
                if ss == s:
                    dp_group = g
    if stages > 1:
        for dd in range(data_parallel):
            g = dist.new_group([dd * stages, dd * stages + stages - 1])
            if dd == d:
                tied_group = g
    return pp_group, pp_ranks, dp_group, tied_group


class PipelineTrainer:
    """One pipeline stage's trainer: its own flat store and optimizer, 1F1B or GPipe
    schedule, optionally data-parallel over replicas of the pipeline."""

    cuda_graph = False  # stage-to-stage transfers run between the layers
    _graph = None
    last_info = None    # the per-layer statistics stay on their stages

    def __init__(self, model: nn.Module, stages: Optional[int] = None, total_steps: int = 1000,
                 optimizer: str = "adamw", compute_dtype: torch.dtype = torch.float32, device=None,
                 group: Optional[dist.ProcessGroup] = None, skip_nonfinite: bool = False,
                 schedule: str = "1f1b", data_parallel: int = 1):
        from ..optim import FlatParamStore, HybridOptimizer, grad_scale_of, label_adamw_only, label_of
        if schedule not in ("1f1b", "gpipe"):
            raise ValueError(f"unknown pipeline schedule {schedule!r}")
        self.schedule = schedule
        self.dp = max(1, data_parallel)
        if self.dp > 1 or group is None:
            stages = stages or dist.get_world_size() // self.dp
            group, self.ranks, self.dp_group, self.tied_group = pipeline_groups(stages, self.dp)
            self.stages = stages
        else:  # an explicit stage group, no data parallelism
            self.stages = stages or dist.get_world_size(group)
            self.ranks = [dist.get_global_rank(group, s) for s in range(self.stages)]
            self.dp_group = None
            self.tied_group = None
            if model.cfg.tie_embeddings and self.stages > 1:
                self.tied_group = dist.new_group([self.ranks[0], self.ranks[-1]])
        self.group = group
        self.stage = self.ranks.index(dist.get_rank())
        self.dp_rank = dist.get_rank() // self.stages if self.dp > 1 else 0
        self.part = PipelineStage(model, self.stages, self.stage)
        self.cfg = model.cfg
        dev = device or next(model.parameters()).device
        self.device = dev
        label_fn = label_of if optimizer == "hybrid" else label_adamw_only
        tied = self.cfg.tie_embeddings and self.stages > 1 and self.part.last
        # the last stage's copy of the tied embedding sits in its own (unsharded) store:
        # it takes the first stage's update and is left out of the global norm
        own = (lambda n, p: not n.startswith("embed.")) if tied else None
        self.store = FlatParamStore(self.part, label_fn, grad_scale_of, self.dp, self.dp_rank,
                                    compute_dtype=compute_dtype, device=dev, param_filter=own)
        self.opt = HybridOptimizer(self.store, total_steps, reduce_fn=self._sum_all, skip_nonfinite=skip_nonfinite)
        self.comm = None
        if self.dp > 1:
            from .fsdp import NcclShardComm
            self.comm = NcclShardComm(self.store, self.dp_group)
        self.tied_store = self.tied_opt = None
        if tied:
            self.tied_store = FlatParamStore(self.part, label_fn, grad_scale_of, 1, 0, compute_dtype=compute_dtype,
                                             device=dev, param_filter=lambda n, p: n.startswith("embed."))
            self.tied_opt = HybridOptimizer(self.tied_store, total_steps, skip_nonfinite=skip_nonfinite)
            self.tied_opt.schedule = self.opt.schedule
            self.tied_opt.norm_share = 0.0
            self.opt.partners.append(self.tied_opt)
        n_moe = len(self.part.layer_ids)
        self._frac = torch.zeros(max(n_moe, 1), self.cfg.e_routed, device=dev)
        self.global_step = 0
        self._batches: List[Dict[str, torch.Tensor]] = []
        self._loss_sum = torch.zeros((), device=dev)
        self.peak_live = 0  # most micro-batches holding activations at once (last step)

    @property
    def ep_store(self):  # the tied embedding copy saves / restores with the stage's store
        return self.tied_store

    @property
    def ep_opt(self):
        return self.tied_opt

    # ------------------------------------------------------------ plumbing
    def _sum_all(self, t: torch.Tensor) -> torch.Tensor:
        """Norm partials and flags: every rank holds a distinct piece (stage x shard)."""
        dist.all_reduce(t, group=self.group if self.dp == 1 else None)
        return t

    def _peer(self, stage: int) -> int:
        return self.ranks[stage]

    def _send(self, t: torch.Tensor, stage: int) -> None:
        dist.send(t.detach().contiguous(), self._peer(stage), group=self.group)

    def _recv(self, shape, dtype, stage: int) -> torch.Tensor:
        t = torch.empty(shape, dtype=dtype, device=self.device)
        dist.recv(t, self._peer(stage), group=self.group)
        return t

    def _exchange(self, send: torch.Tensor, send_stage: int, shape, dtype, recv_stage: int) -> torch.Tensor:
        """Send ``send`` to one neighbour and receive a tensor from one (the same or the
        other) as a single batched pair."""
        buf = torch.empty(shape, dtype=dtype, device=self.device)
        send = send.detach().contiguous()
        ops = [dist.P2POp(dist.isend, send, self._peer(send_stage), self.group),
               dist.P2POp(dist.irecv, buf, self._peer(recv_stage), self.group)]
        for req in dist.batch_isend_irecv(ops):
            req.wait()
        return buf

    def _aux(self, stats: List[Dict]) -> torch.Tensor:
        from ..training.loss import ROUTER_COLLINEARITY_COEF
        zero = torch.zeros((), device=self.device)
        if not stats:
            return zero
        aux = sum(s["aux_loss"] for s in stats)
        z = sum(s["z_loss"] for s in stats)
        coll = sum(s["router_collinearity"] for s in stats)
        return self.cfg.router_aux_loss_coef * aux + self.cfg.router_z_loss_coef * z + \
            ROUTER_COLLINEARITY_COEF * coll

    def _act_shape(self, b: Dict[str, torch.Tensor]):
        Bsz, L = b["input_ids"].shape
        return (Bsz, L, self.cfg.d_model)

    # ------------------------------------------------------------ stage compute
    def _compute(self, b: Dict[str, torch.Tensor], x_in: Optional[torch.Tensor], train: bool):
        """This stage's layers on one micro-batch.  Returns ``(out, aux, loss part)``: ``out``
        is the activation for the next stage, or (last stage) the scalar to differentiate."""
        from .. import ops
        part, cfg = self.part, self.cfg
        L = b["input_ids"].shape[1]
        if part.first:
            x = part.embed(b["input_ids"], part.compute_dtype)
        else:
            if train:
                x_in.requires_grad_(True)
            x = x_in
        stats: List[Dict] = []
        x = part.run(x, L, stats)
        aux = self._aux(stats) if train else torch.zeros((), device=self.device)
        if train:
            for i, st in enumerate(stats):
                if st.get("assignment_frac") is not None:
                    self._frac[i] += st["assignment_frac"]
        part_loss = aux.detach()
        if part.last:
            h = part.final_norm(x)
            w = part.embed.embedding if cfg.tie_embeddings else part.lm_head.kernel.t()
            s, cnt = ops.cross_entropy(h, b["labels"], w, cfg.label_smoothing)
            ce = s / cnt.clamp_min(1.0)
            return ce + aux, None, part_loss + ce.detach()
        return x, aux, part_loss

    def _backward(self, x_in, out, aux, g) -> Optional[torch.Tensor]:
        """Backward of one kept micro-batch; returns the gradient of its stage input."""
        if self.part.last:
            out.backward()
        else:
            ts, gs = [out], [g]
            if aux is not None and aux.requires_grad:
                ts.append(aux)
                gs.append(torch.ones_like(aux))
            torch.autograd.backward(ts, gs)
        return None if x_in is None else x_in.grad

    # ------------------------------------------------------------ schedules
    def _run_gpipe(self, batches) -> None:
        first, last, s = self.part.first, self.part.last, self.stage
        kept = []
        for b in batches:
            x_in = None if first else self._recv(self._act_shape(b), self.part.compute_dtype, s - 1)
            out, aux, pl = self._compute(b, x_in, True)
            self._loss_sum += pl
            if not last:
                self._send(out, s + 1)
            kept.append((x_in, out, aux))
            self.peak_live = max(self.peak_live, len(kept))
        for x_in, out, aux in kept:
            g = None if last else self._recv(out.shape, out.dtype, s + 1)
            gx = self._backward(x_in, out, aux, g)
            if not first:
                self._send(gx, s - 1)

    def _run_1f1b(self, batches) -> None:
        first, last, s, S = self.part.first, self.part.last, self.stage, self.stages
        M = len(batches)
        warm = min(S - s - 1, M)
        steady = M - warm
        dt = self.part.compute_dtype
        kept: List = []  # (input, output, aux) of the micro-batches awaiting their backward

        def fwd(i, x_in):
            out, aux, pl = self._compute(batches[i], x_in, True)
            self._loss_sum += pl
            kept.append((x_in, out, aux))
            self.peak_live = max(self.peak_live, len(kept))
            return out

        def bwd(g):
            x_in, out, aux = kept.pop(0)
            return self._backward(x_in, out, aux, g)

        for i in range(warm):
            x_in = None if first else self._recv(self._act_shape(batches[i]), dt, s - 1)
            out = fwd(i, x_in)
            if not last:
                self._send(out, s + 1)
        x_in = None
        if steady > 0 and not first:
            x_in = self._recv(self._act_shape(batches[warm]), dt, s - 1)
        for k in range(steady):
            out = fwd(warm + k, x_in)
            # the gradient that comes back belongs to the oldest kept micro-batch
            g = None if last else self._exchange(out, s + 1, kept[0][1].shape, out.dtype, s + 1)
            gx = bwd(g)
            x_in = None
            if first:
                continue
            if k < steady - 1:
                x_in = self._exchange(gx, s - 1, self._act_shape(batches[warm + k + 1]), dt, s - 1)
            else:
                self._send(gx, s - 1)
        while kept:
            g = None if last else self._recv(kept[0][1].shape, dt, s + 1)
            gx = bwd(g)
            if not first:
                self._send(gx, s - 1)

    # ------------------------------------------------------------ micro-step / apply (Trainer interface)
    def micro_step(self, batch: Dict[str, torch.Tensor]):
        """Queue one micro-batch; ``apply`` runs the schedule over the queued ones."""
        self._batches.append(batch)
        return None, {}

    def apply(self, n_accum: Optional[int] = None) -> Dict[str, torch.Tensor]:
        """The schedule over the queued micro-batches, the tied embedding gradient sum, the
        data-parallel gradient reduction, then the optimizer step on this stage's parameters."""
        batches, M = self._batches, max(len(self._batches), 1)
        n = n_accum if n_accum is not None else M
        self._frac.zero_()
        self.peak_live = 0
        self.part.train()
        (self._run_1f1b if self.schedule == "1f1b" else self._run_gpipe)(batches)
        if self.tied_group is not None and (self.part.first or self.part.last):
            st = self.tied_store if self.part.last else self.store
            dist.all_reduce(st.grad_view(st.by_name["embed.embedding"]), group=self.tied_group)
        frac = self._frac / M
        if self.dp > 1:
            dist.all_reduce(frac, group=self.dp_group)
            frac = frac / self.dp
            if self.tied_store is not None:
                dist.all_reduce(self.tied_store.grad, group=self.dp_group)
            self.comm.reduce_scatter_grads()
        out = self.opt.step(n * self.dp, frac)
        if self.comm is not None:
            self.comm.all_gather_params()
        loss = self._loss_sum.clone()
        dist.all_reduce(loss, group=self.group)  # this replica's loss: CE + every layer's terms
        out["loss"] = loss / M
        self.reset_accumulators()
        self.global_step += 1
        return out

    def reset_accumulators(self) -> None:
        self._batches = []
        self._loss_sum = torch.zeros((), device=self.device)
        self.store.zero_grad()
        if self.tied_store is not None:
            self.tied_store.zero_grad()

    def train_step(self, micro_batches: List[Dict[str, torch.Tensor]]) -> Dict[str, torch.Tensor]:
        for b in micro_batches:
            self.micro_step(b)
        return self.apply(len(micro_batches))

    @torch.no_grad()
    def eval_loss(self, batch: Dict[str, torch.Tensor]) -> torch.Tensor:
        self.part.eval()
        s = self.stage
        x_in = None if self.part.first else self._recv(self._act_shape(batch), self.part.compute_dtype, s - 1)
        out, _, _ = self._compute(batch, x_in, False)
        if not self.part.last:
            self._send(out, s + 1)
        loss = out.detach().reshape(()) if self.part.last else torch.zeros((), device=self.device)
        dist.all_reduce(loss, group=self.group)
        self.part.train()
        return loss

    def close(self) -> None:
        pass
