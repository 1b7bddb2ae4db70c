"""The reference's hybrid optimizer and apply step on a ``FlatParamStore``.

Apply step (reference `train_setup.py:490-550`), on the owned shard:

1. ``avg = grad / n_accum``; per-group non-finite flags; ``global_norm`` of
   ``avg``; ``clip_factor`` (logged only).
2. ``nan_to_num(avg)`` -- a non-finite gradient becomes 0 and the update still
   runs (reference behaviour; ``skip_nonfinite=True`` makes it a real skip).
3. gradient x0.2 for ``decay_a``/``A_log``, x0.3 for router tensors.
4. ``clip_by_global_norm(0.35)`` then per-label updates (reference
   `optimizer.py:84-239`):

   * ``muon``: ``-lr*NS3(g) - lr*0.01*p`` with ``lr = 0.008*schedule``,
   * ``lion``: ``-lr*(sign(0.1 g + 0.9 m) + 0.1 p)``, ``m <- 0.01 g + 0.99 m``,
     ``lr = 2e-4*schedule*backoff``,
   * ``adamw_decay`` / ``adamw_nodecay``: optax ``adamw`` (b1 0.9, b2 0.999,
     eps 1e-8, wd 0.01 / 0), ``lr = 6e-4*schedule*backoff``,
   * ``frozen``: no update.
5. parameter clip ``+-100`` + nan_to_num; ``router_temp <- router_temp -
   0.02*(router_temp - 10)``; ``expert_bias += 0.02*sign(1/E - assignment_frac)``
   (overloaded experts go down).
6. ``was_clipped`` is evaluated on the parameters *before* the update.

On CUDA tensors every elementwise piece runs in one fused kernel per step over
the owned segment table (``ops.kernels.optim_apply``); Muon's Newton-Schulz runs
first, two grouped tcgen05 GEMMs per step for all matrices of a tensor
(``ops.kernels.newton_schulz3``).  Cross-rank reductions (norms, flags) go
through ``reduce_fn``.
"""
from __future__ import annotations

from typing import Callable, Dict, Optional

import torch

from .. import ops
from ..ops import reference as R
from .schedule import DIAG_GROUPS, LRSchedule, diag_group_of, path_key, resume_backoff
from .store import FlatParamStore

ROUTER_TEMP_DECAY_RATE = 0.02
ROUTER_TEMP_INIT = 10.0
EXPERT_BIAS_GAMMA = 0.02
GLOBAL_CLIP = 0.35
PARAM_CLIP = 1e2


def _muon_direction(s, g: torch.Tensor, ns) -> torch.Tensor:
    """Newton-Schulz orthogonalisation of a Muon matrix's update.  A tensor-parallel piece
    is orthogonalised as part of its whole matrix: the pieces are all-gathered over the
    tensor-parallel group, every rank runs the iteration on the full matrix and keeps its
    piece (the same direction as without tensor parallelism)."""
    from ..parallel.tp import get_tp, shard_spec, shard_tensor, unshard_tensors
    spec = shard_spec(s.param)
    tp = get_tp()
    if spec is None or tp is None:
        return ns(g)
    import torch.distributed as dist
    parts = [torch.empty_like(g) for _ in range(tp.world)]
    dist.all_gather(parts, g.contiguous(), group=tp.group)
    full = ns(unshard_tensors(parts, spec[0], spec[1]))
    return shard_tensor(full, spec[0], spec[1], tp.world, tp.rank)


class HybridOptimizer:
    def __init__(self, store: FlatParamStore, total_steps: int,
                 reduce_fn: Optional[Callable[[torch.Tensor], torch.Tensor]] = None,
                 skip_nonfinite: bool = False, muon_lr: float = 0.008, lion_lr: float = 2e-4,
                 adamw_lr: float = 6e-4, offload_moments: bool = False):
        self.store = store
        self.schedule = LRSchedule(total_steps)
        self.reduce_fn = reduce_fn or (lambda t: t)
        self.skip_nonfinite = skip_nonfinite
        # called with the step's global is-finite flag after the statistics are reduced and
        # before any parameter moves (every rank calls it at the same point)
        self.before_finish = None
        self.base = {"muon": muon_lr, "lion": lion_lr, "adamw_decay": adamw_lr, "adamw_nodecay": adamw_lr}
        self.count = 0
        dev = store.device
        # ``offload_moments``: the two moments live in (pinned) host memory and each
        # tensor's slice is staged to the device for its update and written back: 8 bytes
        # per parameter leave the GPU for two PCIe copies per step (the update then runs
        # as PyTorch ops, not the fused kernel)
        self.offload = bool(offload_moments)
        host = self.offload and dev.type == "cuda"
        mdev = torch.device("cpu") if host else dev
        self.m = torch.zeros(store.shard, dtype=torch.float32, device=mdev, pin_memory=host)
        self.v = torch.zeros(store.shard, dtype=torch.float32, device=mdev, pin_memory=host)
        self.owned = store.owned()
        self.group_idx = {g: i for i, g in enumerate(DIAG_GROUPS)}
        # (gradient peer table, compute peer table): set by a peer-memory shard comm
        self.peers = None
        # optimizers of further stores stepped together with this one (shared norm / clip)
        self.partners: list = []
        # share of this store's norm statistics in the cross-rank sum (1 / replicas)
        self.norm_share = 1.0

    def uses_kernels(self) -> bool:
        if self.offload:
            return False
        gbuf = self.store.grad
        if not ops.use_cuda(gbuf):
            return False
        from ..ops import kernels as K
        return hasattr(K, "optim_apply")

    # -------------------------------------------------------------- lr values
    def lrs(self, step: int) -> Dict[str, float]:
        s = self.schedule(step)
        b = resume_backoff(step)
        return {"muon": self.base["muon"] * s, "lion": self.base["lion"] * s * b,
                "adamw_decay": self.base["adamw_decay"] * s * b,
                "adamw_nodecay": self.base["adamw_nodecay"] * s * b, "frozen": 0.0}

    def _sl(self, s):
        o = s.offset - self.store.lo
        return slice(o, o + s.numel)

    # -------------------------------------------------------------- the step
    @torch.no_grad()
    def step(self, n_accum: int, assignment_frac: Optional[torch.Tensor] = None) -> Dict[str, torch.Tensor]:
        """One optimizer step.  ``partners`` (optimizers of other parameter stores,
        e.g. the expert-parallel experts) share the global norm, the clip coefficient
        and the non-finite flags with this one: their statistics are added to this
        optimizer's before the single cross-rank reduction."""
        ng = len(DIAG_GROUPS)
        # one small vector reduced across ranks: [sumsq(avg), sumsq(g), was_clipped, flags...]
        red = torch.zeros(3 + ng, dtype=torch.float32, device=self.store.device)
        self._prepare(n_accum, red)
        for p in self.partners:
            p._prepare(n_accum, red)
        red = self.reduce_fn(red)
        global_norm = red[0].sqrt()
        is_finite = torch.isfinite(global_norm)
        clip_norm = red[1].sqrt()
        coef = torch.where(clip_norm < GLOBAL_CLIP, torch.ones_like(clip_norm), GLOBAL_CLIP / clip_norm)
        if self.before_finish is not None:
            self.before_finish(is_finite)  # e.g. the pre-apply snapshot of a non-finite step
        if self.skip_nonfinite and not bool(is_finite):
            return self._info(global_norm, is_finite, red, skipped=True)
        for opt in [self] + list(self.partners):
            opt._finish(coef, assignment_frac)
        return self._info(global_norm, is_finite, red, skipped=False)

    def _prepare(self, n_accum: int, red: torch.Tensor) -> None:
        """Average, non-finite flags, nan_to_num, per-tensor gradient scales and both
        squared norms of the owned gradients, added into ``red``."""
        st = self.store
        gbuf = st.grad[st.lo:st.hi]
        inv = 1.0 / float(n_accum)
        if self.uses_kernels():
            from ..ops import kernels as K
            part = torch.zeros_like(red)
            K.optim_prepare(self, inv, part)
            red[0:2] += part[0:2] * self.norm_share
            red[2:] = torch.maximum(red[2:], part[2:])
            return
        for s in self.owned:
            if not s.param.requires_grad:
                continue
            sl = self._sl(s)
            avg = gbuf[sl].float() * inv
            red[0] += avg.double().square().sum().float() * self.norm_share
            if not torch.isfinite(avg).all():
                red[3 + self.group_idx[diag_group_of(s.name)]] = 1.0
            g = torch.nan_to_num(avg, nan=0.0, posinf=0.0, neginf=0.0) * s.grad_scale
            gbuf[sl] = g
            red[1] += g.double().square().sum().float() * self.norm_share
        for s in self.owned:
            if (st.master_view(s).abs() >= PARAM_CLIP).any():
                red[2] = 1.0

    def _finish(self, coef: torch.Tensor, assignment_frac: Optional[torch.Tensor]) -> None:
        st = self.store
        gbuf = st.grad[st.lo:st.hi]
        use_k = self.uses_kernels()
        lrs = self.lrs(self.count)
        # Muon directions first (matrix-wise), written over the gradient buffer
        if use_k:
            from ..ops import kernels as K
        ns = K.newton_schulz3 if use_k else R.newton_schulz3
        for s in self.owned:
            if s.label == "muon" and s.param.requires_grad:
                sl = self._sl(s)
                g = (gbuf[sl].float() * coef).view(s.shape)
                gbuf[sl] = _muon_direction(s, g, ns).reshape(-1)
        if use_k:
            K.optim_apply(self, lrs, coef, assignment_frac)  # also writes the compute copy
        else:
            self._apply_eager(lrs, coef, gbuf, assignment_frac)
            st.publish_owned()
            if self.offload and self.m.device != st.device:
                # the host moments are read by checkpoints on the host: the write-backs land first
                torch.cuda.current_stream(st.device).synchronize()
        self.count += 1

    def _stage(self, buf: torch.Tensor, sl: slice, dev: torch.device) -> torch.Tensor:
        """The slice of a moment buffer on ``dev`` (a view when it is there already)."""
        t = buf[sl]
        return t if t.device == dev else t.to(dev, non_blocking=True)

    @staticmethod
    def _unstage(buf: torch.Tensor, sl: slice, t: torch.Tensor) -> None:
        if buf.device != t.device:  # stream-ordered: the next stage of this slice follows it
            buf[sl].copy_(t, non_blocking=True)

    def _apply_eager(self, lrs, coef, gbuf, assignment_frac):
        st = self.store
        t = self.count + 1
        bc1 = 1.0 - 0.9 ** t
        bc2 = 1.0 - 0.999 ** t
        bias_idx = 0
        for s in self.owned:
            sl = self._sl(s)
            p = st.master[sl]
            lab = s.label
            lr = lrs[lab]
            if lab == "muon" and s.param.requires_grad:
                p.add_(-lr * gbuf[sl].float() - lr * 0.01 * p)
            elif lab == "lion" and s.param.requires_grad:
                g = gbuf[sl].float() * coef
                m = self._stage(self.m, sl, p.device)
                upd = torch.sign(0.1 * g + 0.9 * m) + 0.1 * p
                m.mul_(0.99).add_(0.01 * g)
                p.add_(-lr * upd)
                self._unstage(self.m, sl, m)
            elif lab.startswith("adamw"):
                g = gbuf[sl].float() * coef if s.param.requires_grad else torch.zeros_like(p)
                m, v = self._stage(self.m, sl, p.device), self._stage(self.v, sl, p.device)
                m.mul_(0.9).add_(0.1 * g)
                v.mul_(0.999).add_(0.001 * g * g)
                upd = (m / bc1) / ((v / bc2).sqrt() + 1e-8)
                if lab == "adamw_decay":
                    upd = upd + 0.01 * p
                p.add_(-lr * upd)
                self._unstage(self.m, sl, m)
                self._unstage(self.v, sl, v)
            p.copy_(torch.nan_to_num(p.clamp(-PARAM_CLIP, PARAM_CLIP), nan=0.0, posinf=PARAM_CLIP,
                                     neginf=-PARAM_CLIP))
            key = path_key(s.name)
            if "router_temp" in key:
                p.sub_(ROUTER_TEMP_DECAY_RATE * (p - ROUTER_TEMP_INIT))
            if "expert_bias" in key:
                if assignment_frac is not None:
                    idx = self.bias_index(s)
                    frac = assignment_frac[idx].to(p.device)
                    target = 1.0 / p.numel()
                    p.add_(EXPERT_BIAS_GAMMA * torch.where(frac > target, -1.0, 1.0))
                bias_idx += 1

    def bias_index(self, s) -> int:
        """Row of ``assignment_frac`` for an ``expert_bias`` tensor: order of the
        expert_bias leaves in parameter order (reference
        ``_build_expert_bias_index_map``, `train_setup.py:232-262`)."""
        if not hasattr(self, "_bias_rows"):
            rows = [x.name for x in self.store.segs if "expert_bias" in path_key(x.name)]
            self._bias_rows = {n: i for i, n in enumerate(rows)}
        return self._bias_rows[s.name]

    def _info(self, global_norm, is_finite, red, skipped):
        safe = torch.where(is_finite, global_norm, torch.ones_like(global_norm))
        clip_factor = torch.where(is_finite, torch.clamp(1.0 / (safe + 1e-6), max=1.0), torch.zeros_like(safe))
        return {"global_norm": global_norm, "is_finite": is_finite, "clip_factor": clip_factor,
                "group_nonfinite_flags": red[3:] > 0, "was_clipped": red[2] > 0, "skipped": skipped}

    # -------------------------------------------------------------- state io
    def state_dict(self) -> Dict[str, object]:
        return {"count": self.count, "m": self.m, "v": self.v}

    def load_state_dict(self, sd) -> None:
        self.count = int(sd["count"])
        self.m.copy_(sd["m"])
        self.v.copy_(sd["v"])
