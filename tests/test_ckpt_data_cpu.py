"""Checkpoint round trip / graft-merge / torn saves, and the multi-source loader."""
import json
import os

import numpy as np
import torch

from atomic_ai_hybrid_b200 import get_preset
from atomic_ai_hybrid_b200.ckpt import CheckpointManager, load_file
from atomic_ai_hybrid_b200.data import dataloader_multi_source, resolve_source_files
from atomic_ai_hybrid_b200.models import HybridMoEModel
from atomic_ai_hybrid_b200.training.trainer import Trainer


def _trainer(cfg, seed=0):
    torch.manual_seed(seed)
    m = HybridMoEModel(cfg, compute_dtype=torch.float32)
    tr = Trainer(m, total_steps=20, optimizer="hybrid", compute_dtype=torch.float32, device=torch.device("cpu"))
    tr.opt.schedule.warmup = 1
    return tr


def _step(tr, cfg, seed=1):
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, cfg.vocab_size, (2, 65), generator=g)
    tr.train_step([{"input_ids": ids[:, :-1], "labels": ids[:, 1:]}])


def test_checkpoint_round_trip_and_dtypes(tmp_path):
    cfg = get_preset("reference_tiny")
    tr = _trainer(cfg)
    _step(tr, cfg)
    mgr = CheckpointManager(str(tmp_path), "latest", max_to_keep=1)
    mgr.save(7, tr, {"epoch": 0, "best_val_loss": 3.0}, asynchronous=True)
    mgr.finalize()
    assert mgr.steps() == [7]
    params = load_file(os.path.join(str(tmp_path), "latest", "7", "params-rank0.safetensors"))
    assert params["block_0/moe/routed_w1"].dtype == torch.bfloat16
    assert params["embed/embedding"].dtype == torch.float32
    assert "block_0/layer_0/sublayer/gdn2/q_proj/kernel" in params
    tr2 = _trainer(cfg, seed=3)
    meta = mgr.restore(7, tr2)
    assert meta["fresh"] == [] and meta["global_step"] == 7 and meta["epoch"] == 0
    for s1, s2 in zip(tr.store.segs, tr2.store.segs):
        a, b = tr.store.master_view(s1), tr2.store.master_view(s2)
        if s1.name.endswith(("routed_w1", "routed_w2")):
            torch.testing.assert_close(b, a.to(torch.bfloat16).float())
        else:
            torch.testing.assert_close(b, a)
    assert tr2.opt.count == tr.opt.count
    torch.testing.assert_close(tr2.opt.m, tr.opt.m)
    # training continues identically after the restore (moments restored exactly)
    _step(tr, cfg, 2)
    _step(tr2, cfg, 2)


def test_graft_merge_and_pruning(tmp_path):
    cfg = get_preset("tiny", num_layers=2, layer_types=("mamba2", "gdn2"))
    tr = _trainer(cfg)
    mgr = CheckpointManager(str(tmp_path), "best_val", max_to_keep=2)
    for s in (1, 2, 3):
        mgr.save(s, tr, {}, asynchronous=False)
    assert mgr.steps() == [2, 3]
    bigger = get_preset("tiny", num_layers=3, layer_types=("mamba2", "gdn2", "gdn2"))
    tr2 = _trainer(bigger)
    meta = mgr.restore(3, tr2)
    assert any(n.startswith("layer_2/") for n in meta["fresh"])
    assert any(n.startswith("layer_0/") for n in meta["restored"])


def test_torn_checkpoint_is_ignored(tmp_path):
    cfg = get_preset("tiny", num_layers=2, layer_types=("mamba2", "gdn2"))
    tr = _trainer(cfg)
    mgr = CheckpointManager(str(tmp_path), "latest", max_to_keep=3)
    mgr.save(1, tr, {}, asynchronous=False)
    mgr.save(2, tr, {}, asynchronous=False)
    os.remove(os.path.join(str(tmp_path), "latest", "2", "COMMIT"))  # crash before commit
    assert mgr.latest_step() == 1
    p = os.path.join(str(tmp_path), "latest", "1", "params-rank0.safetensors")
    with open(p, "r+b") as f:
        f.truncate(os.path.getsize(p) // 2)
    try:
        mgr.restore(1, _trainer(cfg))
        raise AssertionError("truncated checkpoint restored")
    except ValueError:
        pass


def _write_source(d, prefix, n, ctx, base):
    ids = (np.arange(n * ctx, dtype=np.int32).reshape(n, ctx) + base)
    np.save(os.path.join(d, f"{prefix}_input_ids.npy"), ids)
    np.save(os.path.join(d, f"{prefix}_labels.npy"), ids + 1)


def test_loader_modes_split_and_skip(tmp_path):
    d = str(tmp_path)
    _write_source(d, "a", 40, 16, 0)
    _write_source(d, "b", 20, 16, 100000)
    pairs = resolve_source_files(d, "a") + [(*resolve_source_files(d, "b")[0], 0.5)]
    it, val, steps, vsteps = dataloader_multi_source(pairs, batch_size=4, seq_len=8, pin=False)
    assert steps == (40 + 10 - 2) // 4 and vsteps == 0
    b = next(it)
    assert b["input_ids"].shape == (4, 8) and torch.equal(b["labels"], b["input_ids"] + 1)
    # resume skipping reproduces the stream
    it2, _, _, _ = dataloader_multi_source(pairs, batch_size=4, seq_len=8, skip_batches=1, pin=False)
    nxt = next(it)
    assert torch.equal(next(it2)["input_ids"], nxt["input_ids"])
    rr, _, _, _ = dataloader_multi_source(pairs, batch_size=4, seq_len=8, mode="round_robin", pin=False)
    srcs = [next(rr)["_source_idx"] for _ in range(4)]
    assert srcs == [0, 1, 0, 1]
    # rank slicing of the global batch
    r1, _, _, _ = dataloader_multi_source(pairs, batch_size=4, seq_len=8, rank=1, world=2, pin=False)
    full, _, _, _ = dataloader_multi_source(pairs, batch_size=4, seq_len=8, pin=False)
    assert torch.equal(next(r1)["input_ids"], next(full)["input_ids"][2:])
    _ = json
