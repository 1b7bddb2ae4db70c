"""The Hub mirror of the checkpoint slots, against an in-memory stand-in for the Hub:
uploads after each commit keep the newest step of each slot, a job without local
checkpoints resumes from the mirror (model repo or bucket), and relay failures never
stop training."""
import os
import shutil

import pytest

from atomic_ai_hybrid_b200.ckpt import hub
from atomic_ai_hybrid_b200.training.loop import TrainArgs, main_execution

PRESET = dict(num_layers=2, layer_types=("mamba2", "gdn2"), vocab_size=512, d_model=128, n_heads=2, n_heads_ssm=2,
              d_ff=128, n_routed_experts=4, d_state=32)


class FakeHub:
    """Repo files under ``root/repo/<path>``; bucket files under ``root/bucket/<path>``."""

    def __init__(self, root, fail_upload=False):
        self.root, self.fail_upload, self.log = root, fail_upload, []

    def upload_folder(self, folder, repo_id, path_in_repo, message):
        if self.fail_upload:
            raise ConnectionError("no network")
        dst = os.path.join(self.root, "repo", path_in_repo)
        shutil.rmtree(dst, ignore_errors=True)
        shutil.copytree(folder, dst)
        self.log.append(("upload", path_in_repo))

    def list_files(self, repo_id):
        base = os.path.join(self.root, "repo")
        return [os.path.relpath(os.path.join(d, f), base) for d, _, fs in os.walk(base) for f in fs]

    def delete_folder(self, repo_id, path_in_repo):
        shutil.rmtree(os.path.join(self.root, "repo", path_in_repo))
        self.log.append(("delete", path_in_repo))

    def snapshot(self, repo_id, pattern, local_dir):
        slot = pattern.split("/")[0]
        src = os.path.join(self.root, "repo", slot)
        if os.path.isdir(src):
            shutil.copytree(src, os.path.join(local_dir, slot))

    def sync_bucket(self, src, local_dir):
        slot = src.rstrip("/").split("/")[-1]
        shutil.copytree(os.path.join(self.root, "repo", slot), local_dir, dirs_exist_ok=True)


def _args(ck, **kw):
    a = TrainArgs(preset="tiny", overrides=dict(PRESET), ckpt_root=str(ck), seq_len=64, global_batch=2, accum_steps=1,
                  max_steps=2, eval_every=0, log_every=1, impl="eager", cuda_graph=False, hf_repo_id="me/run",
                  checkpoint_every_s=0.0)
    for k, v in kw.items():
        setattr(a, k, v)
    return a


@pytest.mark.parametrize("source", ["hf_model", "bucket"])
def test_upload_prune_and_resume_from_the_hub(tmp_path, monkeypatch, source):
    fake = FakeHub(str(tmp_path / "hub"))
    monkeypatch.setattr(hub, "_default_api", lambda token: fake)
    s1 = main_execution(_args(tmp_path / "ck1"))
    assert s1["global_step"] == 2
    remote = sorted(os.listdir(tmp_path / "hub" / "repo" / "latest"))
    assert remote == ["2"], remote  # step 1 was uploaded, then pruned
    assert ("upload", "latest/1") in fake.log and ("delete", "latest/1") in fake.log
    # another machine: no local checkpoints, resume from the mirror
    s2 = main_execution(_args(tmp_path / "ck2", max_steps=3, resume_source=source, hf_bucket_id="me/bucket"))
    assert s2["global_step"] == 3 and len(s2["losses"]) == 1
    assert os.listdir(tmp_path / "ck2" / "latest") == ["3"]  # resumed at 2, saved 3, pruned 2


def test_relay_failures_do_not_stop_training(tmp_path, monkeypatch):
    fake = FakeHub(str(tmp_path / "hub"), fail_upload=True)
    monkeypatch.setattr(hub, "_default_api", lambda token: fake)
    s = main_execution(_args(tmp_path / "ck", resume_source="hf_model"))
    assert s["global_step"] == 2 and s["stop_reason"] is None
    assert os.path.exists(tmp_path / "ck" / "latest" / "2" / "COMMIT")


def test_no_relay_without_a_repo(monkeypatch):
    monkeypatch.delenv("HF_REPO_ID", raising=False)
    assert hub.HubRelay.create(None) is None
