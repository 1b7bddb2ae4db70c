"""Training entry point (the reference's ``train.py``).

Example (one GPU):   python train.py --preset hybrid_1b --seq-len 4096 --global-batch 32 --accum-steps 8
Example (8 GPUs):    torchrun --standalone --nproc-per-node 8 train.py --preset hybrid_1b ...
Long context:        torchrun --standalone --nproc-per-node 8 train.py --preset hybrid_long --tp 8 --ep 8 \
                         --seq-len 32768 --global-batch 8 ...
Data: ``--data-dir DIR --data-prefix NAME[:FRACTION] ...`` reads the reference's
``.npy`` token files; without data arguments the run uses synthetic tokens.
"""
import argparse
import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

from atomic_ai_hybrid_b200.training.loop import TrainArgs, main_execution  # noqa: E402


def parse(argv=None) -> TrainArgs:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--preset", default="tiny")
    ap.add_argument("--config", dest="config_yaml", default=None,
                    help="YAML {preset:, overrides:, train:} (atomic_ai_hybrid_b200/configs/)")
    ap.add_argument("--set", action="append", default=[], help="config override key=value (repeatable)")
    ap.add_argument("--ckpt-root", default="checkpoints")
    ap.add_argument("--data-dir", default=None)
    ap.add_argument("--data-prefix", action="append", default=[], help="NAME or NAME:FRACTION")
    ap.add_argument("--data-mode", default="mixed", choices=["mixed", "sequential", "round_robin"])
    ap.add_argument("--seq-len", type=int, default=512)
    ap.add_argument("--global-batch", type=int, default=8)
    ap.add_argument("--accum-steps", type=int, default=1)
    ap.add_argument("--epochs", type=int, default=1)
    ap.add_argument("--max-steps", type=int, default=None)
    ap.add_argument("--total-steps", type=int, default=None)
    ap.add_argument("--optimizer", default="hybrid", choices=["hybrid", "adamw"])
    ap.add_argument("--eval-every", type=int, default=1000)
    ap.add_argument("--log-every", type=int, default=10)
    ap.add_argument("--checkpoint-every-s", type=float, default=95 * 60)
    ap.add_argument("--session-budget-s", type=float, default=9 * 3600 - 300)
    ap.add_argument("--eval-batches", type=int, default=20, help="batches per partial validation")
    ap.add_argument("--early-stop-patience", type=int, default=5)
    ap.add_argument("--val-split", type=float, default=0.05)
    ap.add_argument("--dataset-fraction", type=float, default=1.0, help="global subsample of the sources")
    ap.add_argument("--no-resume", action="store_true")
    ap.add_argument("--resume-slot", default="latest")
    ap.add_argument("--hf-repo-id", default=None, help="mirror checkpoints to this Hub model repo ($HF_REPO_ID)")
    ap.add_argument("--hf-bucket-id", default=None, help="Hub storage bucket to resume from")
    ap.add_argument("--resume-source", default="local_only", choices=["local_only", "hf_model", "bucket"],
                    help="where a resume looks when no local checkpoint exists")
    ap.add_argument("--wandb-project", default=None)
    ap.add_argument("--impl", default="cuda", choices=["cuda", "eager"])
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--skip-nonfinite", action="store_true")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--tp", type=int, default=1, help="tensor-parallel group size (heads split, tokens split "
                                                        "between the mixers)")
    ap.add_argument("--ep", type=int, default=1,
                    help="expert-parallel group size (== --tp with --tp; otherwise any size dividing the world, "
                         "world / ep replicas)")
    ap.add_argument("--remat", action="store_true", help="recompute each layer in the backward (long context)")
    ap.add_argument("--offload-local-moments", action="store_true",
                    help="AdamW moments of expert blocks / tensor-parallel pieces in host memory")
    ap.add_argument("--expert-grad-bf16", action="store_true",
                    help="bf16 gradient accumulators for the expert-parallel experts")
    ap.add_argument("--cp", type=int, default=1,
                    help="context-parallel group size (sequence segments); world / cp data-parallel replicas")
    ap.add_argument("--pp", type=int, default=1,
                    help="pipeline stages (layer blocks); world / pp data-parallel replicas of the pipeline")
    ap.add_argument("--pp-schedule", default="1f1b", choices=("1f1b", "gpipe"))
    ap.add_argument("--reset-router", action="store_true", help="re-draw the routers after a restore")
    a = ap.parse_args(argv)
    over = {}
    for kv in a.set:
        k, v = kv.split("=", 1)
        try:
            over[k] = json.loads(v)
        except json.JSONDecodeError:
            over[k] = v
    prefixes, fracs = [], []
    for p in a.data_prefix:
        name, _, fr = p.partition(":")
        prefixes.append(name)
        fracs.append(float(fr) if fr else 1.0)
    return TrainArgs(preset=a.preset, config_yaml=a.config_yaml, overrides=over, ckpt_root=a.ckpt_root,
                     data_dir=a.data_dir, data_prefixes=prefixes, source_fractions=fracs, data_mode=a.data_mode,
                     seq_len=a.seq_len, global_batch=a.global_batch, accum_steps=a.accum_steps, epochs=a.epochs,
                     max_steps=a.max_steps, total_steps=a.total_steps, optimizer=a.optimizer,
                     eval_every=a.eval_every, log_every=a.log_every, checkpoint_every_s=a.checkpoint_every_s,
                     session_budget_s=a.session_budget_s, resume=not a.no_resume, resume_slot=a.resume_slot,
                     wandb_project=a.wandb_project, impl=a.impl, cuda_graph=not a.no_graph,
                     skip_nonfinite=a.skip_nonfinite, seed=a.seed, tensor_parallel=a.tp, expert_parallel=a.ep,
                     remat=a.remat, reset_router=a.reset_router, context_parallel=a.cp,
                     pipeline_parallel=a.pp, pipeline_schedule=a.pp_schedule, hf_repo_id=a.hf_repo_id,
                     hf_bucket_id=a.hf_bucket_id, resume_source=a.resume_source, eval_batches=a.eval_batches,
                     early_stop_patience=a.early_stop_patience, val_split=a.val_split,
                     dataset_fraction=a.dataset_fraction, offload_local_moments=a.offload_local_moments,
                     expert_grad_bf16=a.expert_grad_bf16)


def apply_yaml_train_section(args: TrainArgs, argv=None) -> TrainArgs:
    """A ``--config`` YAML may carry a ``train:`` section (TrainArgs field names); its values
    apply where the command line left the default."""
    if not args.config_yaml:
        return args
    import dataclasses
    import yaml
    with open(args.config_yaml) as f:
        data = yaml.safe_load(f) or {}
    train = data.get("train") or {}
    defaults = parse([])
    names = {f.name for f in dataclasses.fields(TrainArgs)}
    for k, v in train.items():
        if k not in names:
            raise ValueError(f"{args.config_yaml}: unknown train field {k!r}")
        if getattr(args, k) == getattr(defaults, k):
            setattr(args, k, v)
    return args


if __name__ == "__main__":
    out = main_execution(apply_yaml_train_section(parse()))
    if int(os.environ.get("RANK", "0")) == 0:
        print(json.dumps({k: v for k, v in out.items() if k != "losses"}))
