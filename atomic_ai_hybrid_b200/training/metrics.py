"""Per-step training metrics and their console lines (reference `train.py:1086-1186`).

``step_metrics`` turns the last micro-step's auxiliary statistics (``training.loss``:
per-layer tensors) into the reference's W&B keys -- ``train/*``, and the router health
summaries ``moe/*`` (utilisation spread, temperatures, router column norms, router
collinearity, pre-clip logits, token norms, dropped ratio) -- the indented console
lines that go with them, and the alerts the reference raises (a router column near
collapse, collinear routers).  It reads the statistics on the host, so the loop calls
it on logging steps only.
"""
from __future__ import annotations

from typing import Dict, List, Optional, Tuple

import numpy as np
import torch

MIN_COL_NORM_ALERT = 1e-3     # router column near-collapse
MAX_COS_ALERT = 0.85          # routers of one layer nearly collinear
LOGIT_FAR_PAST_CLIP = 12.0    # router logits clip at +-8


def _host(x) -> Optional[np.ndarray]:
    if x is None:
        return None
    if isinstance(x, torch.Tensor):
        return x.detach().float().cpu().numpy()
    return np.asarray(x, dtype=np.float64)


def step_metrics(step: int, loss: float, aux: Optional[Dict], best_train: float, tokens_per_sec: float,
                 epoch: int, num_experts: int) -> Tuple[Dict[str, float], List[str], List[Tuple[str, str]]]:
    """Returns ``(metrics, console lines, alerts as (title, text))``."""
    m: Dict[str, float] = {"train/loss": loss, "train/best_train_loss": best_train,
                           "train/tokens_per_sec": tokens_per_sec, "train/epoch": epoch}
    lines: List[str] = []
    alerts: List[Tuple[str, str]] = []
    if not aux:
        return m, lines, alerts
    for k in ("ce_loss", "aux_loss", "z_loss"):
        if aux.get(k) is not None:
            m[f"train/{k}"] = float(_host(aux[k]).reshape(-1)[0])
    util = _host(aux.get("expert_utilization"))
    if util is not None:
        std = np.atleast_2d(util).std(axis=-1)
        w = int(std.argmax())
        m["moe/expert_util_std_max"] = float(std[w])
        m["moe/expert_util_std_worst_layer"] = w
        lines.append(f"expert utilization std (max over layers, layer {w}): {std[w]:.4f} | ideal ~= 0, "
                     f"uniform = 1/{max(num_experts - 1, 1)}")
    rt = _host(aux.get("router_temp"))
    if rt is not None:
        rt = np.atleast_1d(rt).reshape(-1)
        w = int(rt.argmax())
        m.update({"moe/router_temp_mean": float(rt.mean()), "moe/router_temp_min": float(rt.min()),
                  "moe/router_temp_max": float(rt.max()), "moe/router_temp_worst_layer": w})
        m.update({f"moe/router_temp_layer{i}": float(v) for i, v in enumerate(rt)})
        lines.append(f"router_temp: mean={rt.mean():.4f} min={rt.min():.4f} max={rt.max():.4f} (worst_layer={w})")
    cn = _host(aux.get("min_col_norm"))
    if cn is not None:
        cn = np.atleast_1d(cn).reshape(-1)
        w = int(cn.argmin())
        m["moe/min_col_norm_worst"] = float(cn[w])
        lines.append(f"min router column norm (min over layers, layer {w}): {cn[w]:.6f}  (watch for drift toward 0)")
        if cn[w] < MIN_COL_NORM_ALERT:
            lines.append(f"[MOE-DIAG] router column near-collapse on layer {w} at global_step={step}: "
                         f"min_col_norm={cn[w]:.6e}")
            alerts.append(("Router column near-collapse",
                           f"layer={w} min_col_norm={cn[w]:.6e} at global_step={step}."))
    mc = _host(aux.get("router_max_cos_per_layer"))
    if mc is not None:
        mc = np.atleast_1d(mc).reshape(-1)
        w = int(mc.argmax())
        m["moe/router_max_cos_worst"] = float(mc[w])
        lines.append(f"router_max_cos (max over layers, layer {w}): {mc[w]:.4f}")
        if mc[w] > MAX_COS_ALERT:
            alerts.append(("Router collinearity high", f"layer={w} max_cos={mc[w]:.4f} at step={step}"))
    lg = _host(aux.get("max_abs_logit_preclip"))
    if lg is not None:
        lg = np.atleast_1d(lg).reshape(-1)
        w = int(lg.argmax())
        m["moe/max_abs_logit_preclip_worst"] = float(lg[w])
        lines.append(f"max|router logit| pre-clip (max over layers, layer {w}): {lg[w]:.3f}  (clip is at +-8)")
        if lg[w] > LOGIT_FAR_PAST_CLIP:
            lines.append(f"[MOE-DIAG] router logits far past clip on layer {w} at global_step={step}: "
                         f"max|logit|={lg[w]:.3f} (clip=+-8)")
    if aux.get("norm_x_mean") is not None:
        mean_all = float(_host(aux["norm_x_mean"]).mean())
        max_all = float(_host(aux["norm_x_max"]).max())
        min_all = float(_host(aux["norm_x_min"]).min())
        m.update({"moe/norm_x_mean": mean_all, "moe/norm_x_max": max_all, "moe/norm_x_min": min_all})
        lines.append(f"||x|| (L2 norm per token): mean={mean_all:.3f}, max={max_all:.3f}, min={min_all:.3f}")
    dr = _host(aux.get("moe_dropped_ratio"))
    if dr is not None:
        dr = np.atleast_1d(dr).reshape(-1)
        w = int(dr.argmax())
        m["moe/dropped_ratio_max"] = float(dr[w])
        lines.append(f"moe dropped_ratio (max over layers, layer {w}): {dr[w]:.4f}  (ideal ~= 0 after warmup)")
    return m, lines, alerts


def model_metrics(model: torch.nn.Module) -> Dict[str, float]:
    """``model/total_params`` and ``model/weights_gb`` (parameters this rank builds)."""
    n = sum(p.numel() for p in model.parameters())
    b = sum(p.numel() * p.element_size() for p in model.parameters())
    return {"model/total_params": float(n), "model/weights_gb": b / 1e9}
