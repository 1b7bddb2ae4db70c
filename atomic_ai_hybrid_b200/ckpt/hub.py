"""Mirror of the checkpoint slots on the Hugging Face Hub (reference
`checkpointing.py:205-319`, used by `train.py:201-215,372-385,797-809,1048`).

* ``upload(slot_dir, slot, step)``: the committed step folder goes to
  ``{repo}/{slot}/{step}``; then every older step of that slot in the repo beyond the
  newest ``keep_last_n`` is deleted.  Called by rank 0 after a checkpoint commits (from
  the checkpoint writer thread, so training does not wait on the network).
* ``download(slot_dir, slot)``: with ``source="hf_model"`` the slot's files of the model
  repo, with ``source="bucket"`` the slot of an HF storage bucket
  (``hf://buckets/{bucket}/{slot}``), are fetched and their step folders placed in the
  local slot directory; returns the newest step, None when there is none.

Like the reference, a relay failure never stops training: errors are printed and the
call returns ``False`` / ``None``.  The network side is an adapter over
``huggingface_hub`` (``_HubApi``); tests substitute an in-memory one.
"""
from __future__ import annotations

import os
import re
import shutil
import tempfile
from typing import Optional


class _HubApi:
    """The few ``huggingface_hub`` calls the relay makes."""

    def __init__(self, token: Optional[str] = None):
        import huggingface_hub as hh  # type: ignore
        self.hh = hh
        self.api = hh.HfApi(token=token)
        self.token = token

    def upload_folder(self, folder: str, repo_id: str, path_in_repo: str, message: str) -> None:
        self.api.create_repo(repo_id, repo_type="model", exist_ok=True)
        self.api.upload_folder(folder_path=folder, repo_id=repo_id, repo_type="model", path_in_repo=path_in_repo,
                               commit_message=message)

    def list_files(self, repo_id: str):
        return self.api.list_repo_files(repo_id, repo_type="model")

    def delete_folder(self, repo_id: str, path_in_repo: str) -> None:
        self.api.delete_folder(path_in_repo=path_in_repo, repo_id=repo_id, repo_type="model")

    def snapshot(self, repo_id: str, pattern: str, local_dir: str) -> None:
        self.hh.snapshot_download(repo_id=repo_id, repo_type="model", allow_patterns=[pattern], local_dir=local_dir,
                                  token=self.token)

    def sync_bucket(self, src: str, local_dir: str) -> None:
        self.hh.sync_bucket(src, local_dir)


def _default_api(token: Optional[str]):
    return _HubApi(token)


class HubRelay:
    def __init__(self, repo_id: Optional[str], api=None, bucket_id: Optional[str] = None, keep_last_n: int = 1):
        self.repo_id, self.api, self.bucket_id, self.keep_last_n = repo_id, api, bucket_id, keep_last_n

    @classmethod
    def create(cls, repo_id: Optional[str] = None, bucket_id: Optional[str] = None,
               keep_last_n: int = 1) -> Optional["HubRelay"]:
        """A relay for ``repo_id`` (default ``$HF_REPO_ID``) with the token ``$HF_TOKEN``;
        None when no repo or bucket is named or ``huggingface_hub`` is missing."""
        repo_id = repo_id or os.environ.get("HF_REPO_ID")
        if not repo_id and not bucket_id:
            return None
        try:
            api = _default_api(os.environ.get("HF_TOKEN"))
        except ImportError:
            print("[HF] huggingface_hub is not installed: checkpoints stay local", flush=True)
            return None
        return cls(repo_id, api, bucket_id, keep_last_n)

    # ------------------------------------------------------------ upload
    def upload(self, slot_dir: str, slot: str, step: int, message: str = "") -> bool:
        step_dir = os.path.join(slot_dir, str(step))
        if not self.repo_id or not os.path.exists(os.path.join(step_dir, "COMMIT")):
            return False
        try:
            self.api.upload_folder(step_dir, self.repo_id, f"{slot}/{step}", f"[{slot}] step {step} {message}".strip())
            print(f"[HF] uploaded {slot}/{step}", flush=True)
        except Exception as e:
            print(f"[HF] upload of {slot}/{step} failed: {e!r}", flush=True)
            return False
        try:
            steps = set()
            for path in self.api.list_files(self.repo_id):
                m = re.match(rf"^{re.escape(slot)}/(\d+)/", path)
                if m:
                    steps.add(int(m.group(1)))
            for old in sorted(steps, reverse=True)[self.keep_last_n:]:
                try:
                    self.api.delete_folder(self.repo_id, f"{slot}/{old}")
                except Exception as e:
                    print(f"[HF] could not delete {slot}/{old}: {e!r}", flush=True)
        except Exception as e:
            print(f"[HF] could not list {slot} for pruning: {e!r}", flush=True)
        return True

    # ------------------------------------------------------------ download
    def download(self, slot_dir: str, slot: str, source: str = "hf_model") -> Optional[int]:
        if source not in ("hf_model", "bucket"):
            raise ValueError(f"unknown resume source {source!r} (hf_model | bucket | local_only)")
        os.makedirs(slot_dir, exist_ok=True)
        try:
            if source == "bucket":
                if not self.bucket_id:
                    raise ValueError("resume from a bucket needs a bucket id")
                self.api.sync_bucket(f"hf://buckets/{self.bucket_id}/{slot}", slot_dir)
            else:
                with tempfile.TemporaryDirectory(dir=os.path.dirname(os.path.abspath(slot_dir))) as tmp:
                    self.api.snapshot(self.repo_id, f"{slot}/**", tmp)
                    src = os.path.join(tmp, slot)
                    for name in os.listdir(src) if os.path.isdir(src) else []:
                        dst = os.path.join(slot_dir, name)
                        if name.isdigit() and not os.path.exists(dst):
                            shutil.move(os.path.join(src, name), dst)
        except Exception as e:
            print(f"[HF] download of slot {slot!r} ({source}) failed: {e!r}", flush=True)
            return None
        steps = [int(d) for d in os.listdir(slot_dir)
                 if d.isdigit() and os.path.exists(os.path.join(slot_dir, d, "COMMIT"))]
        if steps:
            print(f"[HF] slot {slot!r}: step {max(steps)}", flush=True)
        return max(steps) if steps else None
