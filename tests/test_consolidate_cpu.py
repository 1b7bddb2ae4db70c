"""Consolidating a multi-rank checkpoint step: expert blocks and tensor-parallel pieces
(any cut) are assembled into whole tensors; the result restores into one process."""
import json
import os

import pytest
import torch

from atomic_ai_hybrid_b200.ckpt.consolidate import consolidate
from atomic_ai_hybrid_b200.ckpt.safetensors_io import load_file, save_file
from atomic_ai_hybrid_b200.parallel.tp import shard_tensor


def _write_step(root, step, per_rank):
    d = os.path.join(root, "latest", str(step))
    os.makedirs(d)
    for r, (params, moments) in enumerate(per_rank):
        save_file(params, os.path.join(d, f"params-rank{r}.safetensors"), {"format": "atomic_ai_hybrid_b200/params"})
        save_file(moments, os.path.join(d, f"opt-rank{r}.safetensors"), {"format": "atomic_ai_hybrid_b200/opt"})
    with open(os.path.join(d, "metadata.json"), "w") as f:
        json.dump({"global_step": step, "opt_count": 3, "world": len(per_rank)}, f)
    with open(os.path.join(d, "COMMIT"), "w") as f:
        f.write(str(step))


def test_expert_blocks_and_tp_pieces_become_whole(tmp_path):
    g = torch.Generator().manual_seed(0)
    experts = torch.randn(8, 16, 32, generator=g)        # routed experts, split 4 + 4
    qkv = torch.randn(64, 96, generator=g)                # a fused projection cut in 3 blocks, then 2 ways
    rep = torch.randn(64, generator=g).to(torch.bfloat16)
    name_e, name_q, name_r = "block_0/moe/routed_w1", "block_0/gdn2/qkv/kernel", "final_norm/scale"
    ranks = []
    for r in range(2):
        pq = shard_tensor(qkv, 1, 3, 2, r)
        params = {f"{name_e}#experts[{4 * r}:{4 * r + 4}]": experts[4 * r:4 * r + 4],
                  f"{name_q}#tp[{r}/2,d1p3]": pq}
        moments = {f"mu/{name_q}#tp[{r}/2,d1p3]": 2 * pq, f"nu/{name_q}#tp[{r}/2,d1p3]": 3 * pq}
        if r == 0:
            params[name_r] = rep
        ranks.append((params, moments))
    _write_step(str(tmp_path / "in"), 7, ranks)
    info = consolidate(str(tmp_path / "in"), "latest", 7, str(tmp_path / "out"))
    assert info["params"] == 3 and info["moments"] == 2 and info["moments_incomplete"] == []
    d = tmp_path / "out" / "latest" / "7"
    p = load_file(str(d / "params-rank0.safetensors"))
    assert torch.equal(p[name_e], experts) and torch.equal(p[name_q], qkv) and torch.equal(p[name_r], rep)
    m = load_file(str(d / "opt-rank0.safetensors"))
    assert torch.equal(m[f"nu/{name_q}"], 3 * qkv)
    meta = json.loads((d / "metadata.json").read_text())
    assert meta["world"] == 1 and meta["opt_count"] == 3 and (d / "COMMIT").exists()


def test_incomplete_step_is_refused(tmp_path):
    e = torch.zeros(4, 2)
    _write_step(str(tmp_path / "in"), 1, [({"w#experts[0:4]": e, "v#experts[4:8]": e}, {})])
    with pytest.raises(ValueError, match="does not cover"):
        consolidate(str(tmp_path / "in"), "latest", 1, str(tmp_path / "out"))
