"""The reference's checkpoint tree (flax parameter paths, optax chain state with masked
per-label AdamW moments) converts into this framework's layout and restores into the
model with nothing left at its fresh initialisation."""
import collections

import numpy as np
import torch

from atomic_ai_hybrid_b200 import get_preset
from atomic_ai_hybrid_b200.ckpt.manager import CheckpointManager
from atomic_ai_hybrid_b200.ckpt.orbax_convert import convert_tree
from atomic_ai_hybrid_b200.models import HybridMoEModel
from atomic_ai_hybrid_b200.models.hybrid import flax_path
from atomic_ai_hybrid_b200.training.trainer import Trainer

ScaleByAdamState = collections.namedtuple("ScaleByAdamState", "count mu nu")
MaskedState = collections.namedtuple("MaskedState", "inner_state")


def _nest(flat):
    tree = {}
    for path, v in flat.items():
        node = tree
        parts = path.split("/")
        for p in parts[:-1]:
            node = node.setdefault(p, {})
        node[parts[-1]] = v
    return tree


def test_reference_tree_converts_and_restores(tmp_path):
    cfg = get_preset("reference_tiny", dropout_rate=0.0)
    torch.manual_seed(1)
    src = HybridMoEModel(cfg, compute_dtype=torch.float32)
    flat = {flax_path(n): p.detach().numpy().copy() for n, p in src.named_parameters()}
    rng = np.random.RandomState(0)
    mu = {k: np.asarray(rng.randn(*v.shape), dtype=np.float32) for k, v in flat.items()}
    nu = {k: np.asarray(np.abs(rng.randn(*v.shape)), dtype=np.float32) for k, v in flat.items()}
    # two labels, each holding the moments of half of the parameters (the rest masked out)
    keys = sorted(flat)
    half = set(keys[::2])
    empty = np.zeros((0,), np.float32)

    def masked(src_tree, take):
        return _nest({k: (v if (k in half) == take else empty) for k, v in src_tree.items()})

    inner = {"adamw_decay": MaskedState(ScaleByAdamState(np.array(7), masked(mu, True), masked(nu, True))),
             "adamw_nodecay": MaskedState(ScaleByAdamState(np.array(7), masked(mu, False), masked(nu, False)))}
    tree = {"params": {"params": _nest(flat)}, "opt_state": ({}, {"inner_states": inner})}
    info = convert_tree(tree, str(tmp_path), 12, metadata={"global_step": 12, "epoch": 1})
    assert info["params"] == len(flat) and info["moments"] == 2 * len(flat) and info["opt_count"] == 7

    torch.manual_seed(2)
    dst = HybridMoEModel(cfg, compute_dtype=torch.float32)
    tr = Trainer(dst, total_steps=10, optimizer="adamw", compute_dtype=torch.float32, device=torch.device("cpu"))
    meta = CheckpointManager(str(tmp_path)).restore(12, tr)
    assert meta["fresh"] == [] and len(meta["restored"]) == len(flat)
    assert meta["epoch"] == 1 and tr.opt.count == 7
    for n, p in dst.named_parameters():
        ref = torch.from_numpy(flat[flax_path(n)])
        if "routed_w" in n:  # stored in bf16, as the reference does
            ref = ref.to(torch.bfloat16).float()
        assert torch.equal(p.detach().float(), ref), n
    st = tr.store
    for s in st.segs:
        o = s.offset - st.lo
        k = flax_path(s.name)
        assert torch.equal(tr.opt.m[o:o + s.numel].view(s.shape), torch.from_numpy(mu[k])), k
        assert torch.equal(tr.opt.v[o:o + s.numel].view(s.shape), torch.from_numpy(nu[k])), k
