"""``make_shard_and_compile`` with the reference's return contract
(reference `train_setup.py:368-636`), built from this framework's pieces.

Returns ``(micro_step, apply_step, val_step, ctx, optimizer, model, store,
trainer, data_slice, lr_schedule)``: ``micro_step(batch)`` runs one forward/
backward into the gradient accumulators, ``apply_step(n_accum, frac)`` the
sharded optimizer step with the reference's hooks, ``val_step(batch)`` the
deterministic loss; ``ctx`` is the parallel context (the reference's mesh),
``store`` the flat parameter store (shardings), ``data_slice(r)`` the row range
of rank ``r`` in a global batch."""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..config import ModelConfig
from ..models import HybridMoEModel
from ..parallel.context import get_parallel_context
from .trainer import Trainer


def make_shard_and_compile(config: ModelConfig, total_steps: int, batch_size: int, seq_len: int = 8192,
                           accum_steps: int = 1, optimizer: str = "hybrid", device=None, cuda_graph: bool = True):
    world = dist.get_world_size() if dist.is_available() and dist.is_initialized() else 1
    if batch_size % world:
        raise ValueError(f"batch_size={batch_size} must be divisible by n_devices={world}.")
    device = device or (torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available()
                        else torch.device("cpu"))
    cdt = torch.bfloat16 if device.type == "cuda" else torch.float32
    with torch.device(device):
        model = HybridMoEModel(config, compute_dtype=cdt)
    trainer = Trainer(model, total_steps=total_steps, optimizer=optimizer, compute_dtype=cdt, device=device,
                      cuda_graph=cuda_graph and device.type == "cuda")
    per = batch_size // world

    def data_slice(r: int):
        return slice(r * per, (r + 1) * per)

    return (trainer.micro_step, trainer.apply, trainer.eval_loss, get_parallel_context(), trainer.opt, model,
            trainer.store, trainer, data_slice, trainer.opt.schedule)
