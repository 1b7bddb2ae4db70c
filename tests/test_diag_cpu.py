"""Step diagnostics keep the reference's stdout tags: a non-finite sublayer output
raises ``[FWD-DIAG]``, a large residual ``[RESID-DIAG]``, a non-finite gradient at a
sanitizer ``[BWD-FIX]``, and ``GDN2_FWD_DIAG`` prints the per-stage statistics."""
import torch

from atomic_ai_hybrid_b200 import get_preset
from atomic_ai_hybrid_b200.models import HybridMoEModel
from atomic_ai_hybrid_b200.training.loss import compute_loss
from atomic_ai_hybrid_b200.utils import diag


def _model():
    cfg = get_preset("tiny", num_layers=2, layer_types=("mamba2", "gdn2"), vocab_size=256, d_model=128,
                     n_heads=2, n_heads_ssm=2, d_ff=128, n_routed_experts=4, d_state=32)
    torch.manual_seed(0)
    return HybridMoEModel(cfg, compute_dtype=torch.float32), cfg


def _step(m, cfg):
    ids = torch.randint(0, cfg.vocab_size, (1, 65), generator=torch.Generator().manual_seed(1))
    loss, _ = compute_loss(m, {"input_ids": ids[:, :-1], "labels": ids[:, 1:]})
    loss.backward()
    lines = []
    diag.DIAG.end_step(0, emit=lines.append)
    return lines


def test_clean_step_prints_nothing():
    diag.DIAG.__init__()
    m, cfg = _model()
    assert _step(m, cfg) == []


def test_nonfinite_and_large_residual_are_reported(monkeypatch):
    diag.DIAG.__init__()
    m, cfg = _model()
    with torch.no_grad():
        m.layer_1.sublayer.gdn2.out_proj.kernel[0, 0] = float("nan")
        m.layer_0.sublayer.mamba2.out_proj.kernel.mul_(1e6)
    lines = _step(m, cfg)
    text = "\n".join(lines)
    assert "[FWD-DIAG] non-finite delta: layer=1 type=gdn2" in text
    assert "[RESID-DIAG] current_x after layer=0 type=mamba2" in text
    assert "[BWD-FIX]" in text


def test_stage_diagnostics(monkeypatch):
    monkeypatch.setattr(diag, "STAGES", True)
    diag.DIAG.__init__()
    m, cfg = _model()
    text = "\n".join(_step(m, cfg))
    for tag in ("[MAMBA2-FWD-DIAG] in_proj: all_finite=True", "[MAMBA2-FWD-DIAG] ssd_y",
                "[GDN2-FWD-DIAG] q: all_finite=True", "[GDN2-FWD-DIAG] o"):
        assert tag in text, text
