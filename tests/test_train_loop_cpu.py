"""End-to-end training loop on CPU: checkpoint/resume, fault injection on the host
(NaN gradients -> snapshot + auto-stop, SIGTERM -> emergency save), and a
failing rank among gloo ranks ending the others with an error instead of a hang."""
import json
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp
from _dist import free_port, load_factor, threads_per_rank

from atomic_ai_hybrid_b200.training.loop import TrainArgs, main_execution

PRESET_OVER = dict(num_layers=2, layer_types=("mamba2", "gdn2"), vocab_size=512, d_model=128, n_heads=2,
                   n_heads_ssm=2, d_ff=128, n_routed_experts=4, d_state=32)


def _args(tmp, **kw):
    a = TrainArgs(preset="tiny", overrides=dict(PRESET_OVER), ckpt_root=str(tmp), seq_len=64, global_batch=2,
                  accum_steps=2, max_steps=3, eval_every=0, log_every=1, impl="eager", cuda_graph=False)
    for k, v in kw.items():
        setattr(a, k, v)
    return a


def _write_data(d, cols=65):
    rng = np.random.RandomState(0)
    ids = rng.randint(0, 512, size=(64, cols)).astype(np.int32)
    np.save(os.path.join(d, "src_input_ids.npy"), ids[:, :-1])
    np.save(os.path.join(d, "src_labels.npy"), ids[:, 1:])


def test_checkpoint_and_resume_on_files(tmp_path):
    _write_data(str(tmp_path))
    kw = dict(data_dir=str(tmp_path), data_prefixes=["src"], eval_every=2, eval_batches=2)
    s1 = main_execution(_args(tmp_path / "ck", **kw))
    assert s1["global_step"] == 3 and s1["stop_reason"] is None
    s2 = main_execution(_args(tmp_path / "ck", max_steps=5, **kw))
    assert s2["global_step"] == 5 and len(s2["losses"]) == 2
    assert os.path.exists(tmp_path / "ck" / "latest" / "5" / "COMMIT")
    assert os.path.exists(tmp_path / "ck" / "best_val")


def test_nonfinite_injection_snapshots_and_autostops(tmp_path, monkeypatch):
    monkeypatch.setenv("AHB_INJECT_NAN_STEP", "2-9")
    s = main_execution(_args(tmp_path, max_steps=20))
    assert s["stop_reason"] == "nonfinite" and s["global_step"] == 5
    snap = tmp_path / "nonfinite_snapshots" / "2"
    meta = json.loads((snap / "SNAPSHOT_META.json").read_text())
    assert meta["n_micro"] == 2 and meta["global_step"] == 2
    state = json.loads((snap / "state" / "2" / "metadata.json").read_text())
    # saved before the update of step 2: the optimizer has taken one step
    assert state["tag"] == "NONFINITE_PRE_APPLY" and state["opt_count"] == 1, state
    import torch
    assert torch.load(snap / "rng_rank0.pt")["cpu"].dtype == torch.uint8
    assert os.path.exists(tmp_path / "latest" / "5" / "COMMIT")


def test_sigterm_triggers_emergency_save(tmp_path, monkeypatch):
    monkeypatch.setenv("AHB_INJECT_SIGNAL_STEP", "2")
    s = main_execution(_args(tmp_path, max_steps=10))
    assert s["stop_reason"] == "signal" and s["global_step"] == 2
    meta = json.loads((tmp_path / "latest" / "2" / "metadata.json").read_text())
    assert meta["tag"] == "EMERGENCY_SIGNAL"


def _rank_main(rank, world, port, tmp, pg_timeout_s):
    import torch
    torch.set_num_threads(threads_per_rank(world))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), AHB_PG_TIMEOUT_S=str(pg_timeout_s), AHB_INJECT_RAISE_STEP="2",
                      AHB_INJECT_RAISE_RANK="1")
    try:
        main_execution(_args(tmp, max_steps=5, global_batch=2, accum_steps=1))
    except Exception as e:
        with open(os.path.join(tmp, f"err{rank}.txt"), "w") as f:
            f.write(f"{type(e).__name__}: {e}")
        raise


def test_failing_rank_ends_peers_with_error(tmp_path):
    """Rank 1 raises at step 2; rank 0, waiting in that step's collective, ends with an
    error naming rank 1 and its exception (the notice posted through the store)."""
    port = free_port()
    # the collective timeout bounds how long rank 0 waits in step 2 for the failed rank; under a
    # loaded machine the healthy steps before it are slower, so it scales with the load
    lf = load_factor()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, str(tmp_path), int(20 * lf))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240 * lf)
    assert all(p.exitcode not in (0, None) for p in procs), [p.exitcode for p in procs]
    err0 = (tmp_path / "err0.txt").read_text()
    assert err0.startswith("PeerFailure") and "rank 1 at step 2" in err0 and "injected failure" in err0, err0
    assert "injected failure" in (tmp_path / "err1.txt").read_text()


def test_peer_health_notice_board():
    """The notice board alone: nothing posted -> no failure; a posted failure stops the
    other ranks at their next step check with the failed rank's details."""
    import torch.distributed as dist
    from atomic_ai_hybrid_b200.utils.health import PeerFailure, PeerHealth
    store = dist.HashStore()
    h0, h1, h2 = (PeerHealth(store, r, 3) for r in range(3))
    h0.check(1)
    h1.step = 4
    h1.report(RuntimeError("boom"))
    assert h1.failed_peers() == []  # its own notice is not a peer's
    with pytest.raises(PeerFailure, match="rank 1 at step 4: RuntimeError"):
        h2.check(5)
    assert [f["rank"] for f in h0.failed_peers()] == [1]


def _tp_rank_main(rank, world, port, tmp, ep=1):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), AHB_PG_TIMEOUT_S="60")
    _write_data(tmp)
    out = main_execution(_args(tmp, data_dir=tmp, data_prefixes=["src"], tensor_parallel=2, expert_parallel=ep,
                               max_steps=2, checkpoint_every_s=0.0))
    with open(os.path.join(tmp, f"out{rank}.json"), "w") as f:
        json.dump({k: v for k, v in out.items() if k != "losses"}, f)


@pytest.mark.parametrize("ep", [1, 2])
def test_training_loop_with_tensor_parallelism(tmp_path, ep):
    """train.py's loop with --tp 2 (and --ep 2: experts split over the same ranks) on two
    gloo ranks: both ranks train on the same batches (one data-parallel replica) and the
    checkpoint holds the tensor-parallel pieces."""
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    mp.spawn(_tp_rank_main, args=(2, port, str(tmp_path), ep), nprocs=2, join=True)
    outs = [json.load(open(os.path.join(tmp_path, f"out{r}.json"))) for r in range(2)]
    assert outs[0]["global_step"] == 2 and outs[1]["global_step"] == 2, outs
    from atomic_ai_hybrid_b200.ckpt.safetensors_io import load_file
    root = os.path.join(tmp_path, "latest")
    steps = [d for d in os.listdir(root) if d.isdigit()]
    assert steps, os.listdir(root)
    keys = load_file(os.path.join(root, max(steps, key=int), "params-rank1.safetensors")).keys()
    assert any("#tp[1/2," in k for k in keys), sorted(keys)[:10]


def test_router_reset_touches_only_router_leaves():
    import torch
    from atomic_ai_hybrid_b200 import get_preset
    from atomic_ai_hybrid_b200.models import HybridMoEModel
    from atomic_ai_hybrid_b200.training.router_reset import reset_router
    from atomic_ai_hybrid_b200.training.trainer import Trainer
    cfg = get_preset("tiny", **PRESET_OVER)
    torch.manual_seed(0)
    m = HybridMoEModel(cfg, compute_dtype=torch.float32)
    tr = Trainer(m, total_steps=10, optimizer="adamw", compute_dtype=torch.float32, device=torch.device("cpu"))
    ids = torch.randint(0, cfg.vocab_size, (2, 65))
    tr.train_step([{"input_ids": ids[:, :-1], "labels": ids[:, 1:]}])
    before = {n: p.detach().clone() for n, p in m.named_parameters()}
    m_before, v_before = tr.opt.m.clone(), tr.opt.v.clone()
    changed = reset_router(tr, verbose=False)
    assert sorted(changed) == sorted(n for n in before if n.endswith(".router") or n.endswith("router_temp"))
    for n, p in m.named_parameters():
        if n in changed:
            if n.endswith("router_temp"):
                assert float(p.detach()) == 10.0
            else:
                assert not torch.equal(p, before[n]) and abs(float(p.detach().std()) - 0.02) < 0.01
        else:
            assert torch.equal(p, before[n]), n
    st = tr.store
    for s in st.segs:
        o = s.offset - st.lo
        sl = slice(o, o + s.numel)
        if s.name in changed:
            assert not tr.opt.m[sl].any() and not tr.opt.v[sl].any()
        else:
            assert torch.equal(tr.opt.m[sl], m_before[sl]) and torch.equal(tr.opt.v[sl], v_before[sl])


def _ep_rank_main(rank, world, port, tmp):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), AHB_PG_TIMEOUT_S="60")
    _write_data(tmp)
    out = main_execution(_args(tmp, data_dir=tmp, data_prefixes=["src"], expert_parallel=2, max_steps=2,
                               checkpoint_every_s=0.0, global_batch=world))
    with open(os.path.join(tmp, f"out{rank}.json"), "w") as f:
        json.dump({k: v for k, v in out.items() if k != "losses"}, f)


@pytest.mark.parametrize("world", [2, 4])
def test_training_loop_with_expert_parallelism(tmp_path, world):
    """train.py's loop with --ep 2 on two gloo ranks (all-to-all path), and on four (two
    data-parallel replicas of the expert-parallel pair): it trains and the checkpoint holds
    each rank's block of experts."""
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    mp.spawn(_ep_rank_main, args=(world, port, str(tmp_path)), nprocs=world, join=True)
    outs = [json.load(open(os.path.join(tmp_path, f"out{r}.json"))) for r in range(world)]
    assert all(o["global_step"] == 2 for o in outs), outs
    from atomic_ai_hybrid_b200.ckpt.safetensors_io import load_file
    root = os.path.join(tmp_path, "latest")
    step = max((d for d in os.listdir(root) if d.isdigit()), key=int)
    keys = load_file(os.path.join(root, step, "params-rank1.safetensors")).keys()
    assert any("routed_w1#experts[2:4]" in k for k in keys), sorted(keys)[:10]


def _ep_bf16_rank_main(rank, world, port, tmp, flag):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), AHB_PG_TIMEOUT_S="60")
    import torch
    torch.set_num_threads(threads_per_rank(world))
    _write_data(tmp)
    out = main_execution(_args(tmp, data_dir=tmp, data_prefixes=["src"], expert_parallel=2, max_steps=3,
                               checkpoint_every_s=0.0, global_batch=world, expert_grad_bf16=flag))
    with open(os.path.join(tmp, f"out{rank}.json"), "w") as f:
        json.dump({"losses": [float(x) for x in out["losses"]], "global_step": out["global_step"]}, f)


def test_expert_bf16_gradients_train_like_fp32(tmp_path):
    """--ep 2 with the experts' gradients in bf16 accumulators (a local store of their own):
    three steps with the per-step losses of the fp32-accumulator run (to 2e-2), and the
    checkpoint still holds each rank's block of experts."""
    losses = {}
    for flag in (False, True):
        d = tmp_path / ("bf16" if flag else "fp32")
        d.mkdir()
        port = free_port()
        mp.spawn(_ep_bf16_rank_main, args=(2, port, str(d), flag), nprocs=2, join=True)
        outs = [json.load(open(os.path.join(d, f"out{r}.json"))) for r in range(2)]
        assert all(o["global_step"] == 3 for o in outs), outs
        losses[flag] = outs[0]["losses"]
    assert len(losses[True]) == len(losses[False]) == 3
    for a, b in zip(losses[True], losses[False]):
        assert abs(a - b) <= 2e-2 * abs(b), (losses[True], losses[False])
    from atomic_ai_hybrid_b200.ckpt.safetensors_io import load_file
    root = os.path.join(tmp_path, "bf16", "latest")
    step = max((x for x in os.listdir(root) if x.isdigit()), key=int)
    keys = load_file(os.path.join(root, step, "params-rank1.safetensors")).keys()
    assert any("routed_w1#experts[2:4]" in k for k in keys), sorted(keys)[:10]


def _cp_rank_main(rank, world, port, tmp):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), AHB_PG_TIMEOUT_S="60")
    _write_data(tmp, cols=129)  # segments of 64 tokens: one scan chunk per rank
    out = main_execution(_args(tmp, data_dir=tmp, data_prefixes=["src"], context_parallel=2, max_steps=2,
                               seq_len=128))
    with open(os.path.join(tmp, f"out{rank}.json"), "w") as f:
        json.dump({k: v for k, v in out.items() if k != "losses"}, f)


def test_training_loop_with_context_parallelism(tmp_path):
    """train.py's loop with --cp 2: both ranks read the same batches and hold one half of
    every sequence."""
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    mp.spawn(_cp_rank_main, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    outs = [json.load(open(os.path.join(tmp_path, f"out{r}.json"))) for r in range(2)]
    assert outs[0]["global_step"] == 2 and outs[1]["global_step"] == 2, outs


def _pp_rank_main(rank, world, ports, tmp, stages):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(ports[0]), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), AHB_PG_TIMEOUT_S="60")
    _write_data(tmp)
    kw = dict(data_dir=tmp, data_prefixes=["src"], pipeline_parallel=stages, eval_every=2, eval_batches=1,
              global_batch=2 * (world // stages))
    first = main_execution(_args(tmp, max_steps=2, **kw))
    # the second job gets a rendezvous of its own (the first one's store may still be
    # closing on rank 0 when the other ranks start the second)
    os.environ["MASTER_PORT"] = str(ports[1])
    again = main_execution(_args(tmp, max_steps=3, **kw))  # resumes from the stage files
    with open(os.path.join(tmp, f"out{rank}.json"), "w") as f:
        json.dump({"first": first["global_step"], "again": again["global_step"],
                   "loss": again["losses"][-1] if again.get("losses") else None}, f)


def _free_ports(n):
    socks = []
    for _ in range(n):
        s = socket.socket()
        s.bind(("127.0.0.1", 0))
        socks.append(s)
    ports = [s.getsockname()[1] for s in socks]
    for s in socks:
        s.close()
    return ports


@pytest.mark.parametrize("world,stages", [(2, 2), (4, 2)])
def test_training_loop_with_pipeline_parallelism(tmp_path, world, stages):
    """train.py's loop with --pp 2 (and, on 4 ranks, two data-parallel replicas of the
    pipeline): the stages train, evaluate, checkpoint their own parameters and resume."""
    mp.spawn(_pp_rank_main, args=(world, _free_ports(2), str(tmp_path), stages), nprocs=world, join=True)
    outs = [json.load(open(os.path.join(tmp_path, f"out{r}.json"))) for r in range(world)]
    assert all(o["first"] == 2 and o["again"] == 3 for o in outs), outs
    for d in range(world // stages):  # every stage of a replica reports the replica's whole loss
        rep = outs[d * stages:(d + 1) * stages]
        assert all(o["loss"] == rep[0]["loss"] for o in rep), outs


def test_wandb_run_continues_across_restarts(tmp_path, monkeypatch):
    """With a (fake) wandb installed, the first job writes its run id next to the
    checkpoints and the resumed job continues that run; a fresh start opens a new one."""
    import sys
    import types
    from atomic_ai_hybrid_b200.utils import wandb_logging
    calls = []
    keys = set()

    class _Run:
        def __init__(self, id):
            self.id = id
            self.summary = {}

        def log(self, metrics, step=None):
            calls.append(("log", step))
            keys.update(metrics)

        def finish(self):
            calls.append(("finish", None))

    def init(project=None, config=None, id=None, name=None, resume=None):
        run = _Run(id or f"run{len([c for c in calls if c[0] == 'init'])}")
        calls.append(("init", id))
        return run

    monkeypatch.setitem(sys.modules, "wandb", types.SimpleNamespace(init=init))
    main_execution(_args(tmp_path, max_steps=1, wandb_project="p"))
    assert (tmp_path / "wandb_run_id.txt").read_text() == "run0"
    main_execution(_args(tmp_path, max_steps=2, wandb_project="p"))
    assert [c[1] for c in calls if c[0] == "init"] == [None, "run0"]
    assert any(c == ("log", 2) for c in calls)
    assert {"train/ce_loss", "train/tokens_per_sec", "moe/router_temp_mean", "moe/expert_util_std_max",
            "checkpoint/best_train_loss"} <= keys, sorted(keys)
    main_execution(_args(tmp_path, max_steps=1, wandb_project="p", resume=False))
    assert [c[1] for c in calls if c[0] == "init"][-1] is None
    assert wandb_logging._RUN is None  # finished


def test_step_metrics_follow_the_reference_keys():
    """The router health summaries: keys, worst layers and alerts (collapsed router
    column, collinear routers)."""
    import torch
    from atomic_ai_hybrid_b200.training.metrics import step_metrics
    aux = {"ce_loss": torch.tensor(2.5), "aux_loss": torch.tensor(1.0), "z_loss": torch.tensor(3.0),
           "expert_utilization": torch.tensor([[0.25, 0.25, 0.25, 0.25], [0.7, 0.1, 0.1, 0.1]]),
           "router_temp": torch.tensor([9.0, 10.0]), "min_col_norm": torch.tensor([0.5, 1e-4]),
           "router_max_cos_per_layer": torch.tensor([0.9, 0.1]), "max_abs_logit_preclip": torch.tensor([3.0, 13.0]),
           "norm_x_mean": torch.tensor([1.0, 3.0]), "norm_x_max": torch.tensor([2.0, 5.0]),
           "norm_x_min": torch.tensor([0.5, 0.1]), "moe_dropped_ratio": torch.tensor([0.0, 0.0])}
    m, lines, alerts = step_metrics(7, 2.6, aux, 2.4, 1000.0, 0, 5)
    assert m["train/ce_loss"] == 2.5 and m["train/tokens_per_sec"] == 1000.0
    assert m["moe/expert_util_std_worst_layer"] == 1 and m["moe/router_temp_worst_layer"] == 1
    assert m["moe/router_temp_layer0"] == 9.0 and abs(m["moe/min_col_norm_worst"] - 1e-4) < 1e-9
    assert m["moe/router_max_cos_worst"] == pytest.approx(0.9) and m["moe/norm_x_max"] == 5.0
    assert [t for t, _ in alerts] == ["Router column near-collapse", "Router collinearity high"]
    assert any(line.startswith("[MOE-DIAG] router logits far past clip on layer 1") for line in lines)
    m0, lines0, _ = step_metrics(1, 1.0, None, 1.0, 1.0, 0, 5)
    assert set(m0) == {"train/loss", "train/best_train_loss", "train/tokens_per_sec", "train/epoch"} and not lines0


def test_epoch_end_validation_and_save(tmp_path, capsys):
    """Two passes over a small file source: each epoch ends with the full validation, a
    forced EPOCH_END save and the best-val slot."""
    _write_data(str(tmp_path))
    s = main_execution(_args(tmp_path / "ck", data_dir=str(tmp_path), data_prefixes=["src"], global_batch=8,
                             accum_steps=1, epochs=2, max_steps=None, eval_batches=1))
    out = capsys.readouterr().out
    assert out.count("[EPOCH]") == 4 and "mean validation loss" in out, out[-2000:]
    assert s["global_step"] > 0 and s["best_val"] < float("inf")
    assert os.listdir(tmp_path / "ck" / "best_val")


def _timer_rank(rank, world, port, q):
    import time as _t
    import torch.distributed as dist
    from atomic_ai_hybrid_b200.utils.phase_timer import PhaseTimer
    import torch
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        t = PhaseTimer(torch.device("cpu"))
        for _ in range(2):
            with t.phase("compute"):
                _t.sleep(0.02 * (rank + 1))
            t.end_step()
        q.put((rank, t.report()))
    finally:
        dist.destroy_process_group()


def test_phase_timer_reports_max_over_ranks():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_timer_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    # both ranks report the slower rank's per-step time (40 ms)
    assert got[0] == got[1] and 38.0 < got[0]["compute"] < 80.0, got
