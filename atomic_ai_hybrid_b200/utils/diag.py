"""Step diagnostics with the reference's stdout tags.

The reference prints, from inside the compiled step (``jax.debug.print`` under
``lax.cond``):

* always: ``[FWD-DIAG]`` when a sublayer delta or an MoE output has a non-finite
  value, ``[RESID-DIAG]`` when the residual stream exceeds 1e3 before its clip
  (`model.py:853-875,894-899`), ``[BWD-FIX]`` when a gradient sanitizer met a
  non-finite gradient (`model.py:171-217`);
* with ``GDN2_FWD_DIAG=1``: per-stage ``all_finite`` / ``max_abs`` of the mixers
  (``[MAMBA2-FWD-DIAG]``, ``[GDN2-FWD-DIAG]``; `model.py:104-125`,
  `atomic_ops/kernel_d_pipeline.py:50-91`) and ``[RESID-BREAKDOWN-DIAG]`` when the
  residual or the delta of a layer exceeds 5e2 (`model.py:128-160`).

Here the checks are device reductions folded into one persistent fp32 buffer
(``max`` per slot, in place, so they are captured in the micro-step CUDA graph);
the buffer is copied to pinned host memory once per optimizer step without
stalling the stream and printed one step later.  ``AHB_STEP_DIAG=0`` turns the
always-on checks off.
"""
from __future__ import annotations

import os
from typing import Dict, List, Optional, Tuple

import torch

STAGES = os.environ.get("GDN2_FWD_DIAG", "0") == "1"
ALWAYS = os.environ.get("AHB_STEP_DIAG", "1") == "1"
_CAP = 4096


class Diagnostics:
    def __init__(self):
        self.buf: Optional[torch.Tensor] = None
        self.slots: Dict[Tuple[str, str], int] = {}
        self.order: List[Tuple[str, str]] = []
        self._host = None
        self._ev = None
        self._pending = False

    # ------------------------------------------------------------ recording
    def _slot(self, kind: str, tag: str, device) -> Optional[int]:
        key = (kind, tag)
        i = self.slots.get(key)
        if i is not None:
            return i
        if torch.cuda.is_available() and torch.cuda.is_current_stream_capturing():
            return None  # slots are assigned in eager warm-up iterations before a capture
        if len(self.order) >= _CAP:
            return None
        if self.buf is None or self.buf.device != torch.device(device):
            self.buf = torch.zeros(_CAP, dtype=torch.float32, device=device)
            self.slots, self.order = {}, []
        i = len(self.order)
        self.slots[key] = i
        self.order.append(key)
        return i

    def _put(self, kind: str, tag: str, value: torch.Tensor) -> None:
        i = self._slot(kind, tag, value.device)
        if i is not None:
            torch.maximum(self.buf[i:i + 1], value.reshape(1).float(), out=self.buf[i:i + 1])

    def residual_pair(self, tag: str, device) -> Optional[torch.Tensor]:
        """Two consecutive slots ``[max |x + delta|, delta non-finite]`` that the fused
        residual + RMSNorm kernel folds its statistics into (None when off)."""
        if not ALWAYS:
            return None
        i = self._slot("maxabs", tag, device)
        j = self._slot("nonfinite", tag, device)
        if i is None or j != i + 1:
            return None
        return self.buf[i:i + 2]

    def nonfinite(self, tag: str, t: torch.Tensor) -> None:
        """``[FWD-DIAG]``: set when ``t`` has a NaN or an infinity."""
        if ALWAYS:
            self._put("nonfinite", tag, (~torch.isfinite(t.detach())).any())

    def maxabs(self, tag: str, t: torch.Tensor) -> None:
        """Largest finite magnitude of ``t`` (``[RESID-DIAG]`` above 1e3)."""
        if ALWAYS:
            self._put("maxabs", tag, torch.nan_to_num(t.detach().float(), nan=0.0, posinf=0.0, neginf=0.0)
                      .abs().amax())

    def stage(self, family: str, tag: str, t: torch.Tensor) -> None:
        """``GDN2_FWD_DIAG=1``: all_finite and max_abs of one mixer stage."""
        if STAGES:
            td = t.detach()
            self._put(f"stage_nf:{family}", tag, (~torch.isfinite(td)).any())
            self._put(f"stage_max:{family}", tag,
                      torch.nan_to_num(td.float(), nan=0.0, posinf=0.0, neginf=0.0).abs().amax())

    def resid_breakdown(self, tag: str, before: torch.Tensor, delta: torch.Tensor) -> None:
        if STAGES:
            self._put("rb_before", tag, torch.nan_to_num(before.detach().float(), nan=0.0, posinf=0.0,
                                                         neginf=0.0).abs().amax())
            self._put("rb_delta", tag, torch.nan_to_num(delta.detach().float(), nan=0.0, posinf=0.0,
                                                        neginf=0.0).abs().amax())

    def grad_fixed(self, tag: str, g: torch.Tensor) -> None:
        """``[BWD-FIX]``: a sanitizer met a non-finite incoming gradient."""
        if ALWAYS:
            self._put("bwd_fix", tag, (~torch.isfinite(g)).any())

    # ------------------------------------------------------------ reporting
    def lines(self, vals) -> List[str]:
        out = []
        by = {key: float(vals[i]) for key, i in self.slots.items()}
        for (kind, tag), v in by.items():
            if kind == "nonfinite" and v > 0:
                out.append(f"[FWD-DIAG] non-finite {tag}")
            elif kind == "maxabs" and v > 1e3:
                where = tag.split(": ", 1)[-1]
                out.append(f"[RESID-DIAG] current_x after {where} max|abs|={v:.3e} before sanitization "
                           f"-- residual stream drift")
            elif kind == "bwd_fix" and v > 0:
                out.append(f"[BWD-FIX] non-finite gradient at node {tag} -- sanitized")
            elif kind.startswith("stage_max:"):
                fam = kind.split(":", 1)[1]
                nf = by.get((f"stage_nf:{fam}", tag), 0.0)
                out.append(f"[{fam}-FWD-DIAG] {tag}: all_finite={nf == 0}  max_abs={v:.3e}")
            elif kind == "rb_before":
                d = by.get(("rb_delta", tag), 0.0)
                if max(v, d) > 5e2:
                    out.append(f"[RESID-BREAKDOWN-DIAG] {tag}: current_x_before={v:.3e}  delta={d:.3e}")
        return out

    def end_step(self, step: int, emit=print) -> None:
        """Print the previous step's events (if its copy has landed) and start the
        copy of this step's buffer; then clear it for the next step."""
        if self.buf is None:
            return
        if self._pending and self._ev.query():
            for ln in self.lines(self._host):
                emit(f"{ln} (step {step - 1})")
            self._pending = False
        elif self._pending:
            return  # the last copy is still in flight: keep accumulating into the buffer
        if not self._pending:
            if self.buf.is_cuda:
                if self._host is None:
                    self._host = torch.zeros(_CAP, dtype=torch.float32, pin_memory=True)
                    self._ev = torch.cuda.Event()
                self._host.copy_(self.buf, non_blocking=True)
                self._ev.record()
                self._pending = True
            else:
                for ln in self.lines(self.buf.tolist()):
                    emit(f"{ln} (step {step})")
        self.buf.zero_()


DIAG = Diagnostics()
