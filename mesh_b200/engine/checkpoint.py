"""Checkpoint manager: CBOR checkpoints per job with hash, retention and recovery lookup.

Restates ``agent/src/checkpoint/manager.rs:24-345`` and ``checkpoint/types.rs``: checkpoints live
at ``<checkpoint_dir>/<job_id>/<checkpoint_id>.ckpt`` (the file name the reference uses,
``manager.rs:155``, ``:251``, so either side finds the other's checkpoints); retention keeps at most 5 per job, 10 GB in
total and 24 h of age (``types.rs:35-50``); every checkpoint carries a SHA-256 of its payload that
is verified on load.
"""
from __future__ import annotations

import hashlib
import os
import shutil
import time
import uuid
from dataclasses import asdict, dataclass, field
from pathlib import Path
from typing import List, Optional

import cbor2

# checkpoint file suffix; writes go to "<id>.ckpt.tmp" first and are renamed into place
CKPT_SUFFIX = ".ckpt"


def default_checkpoint_dir() -> Path:
    home = os.environ.get("MESHNET_HOME")
    return (Path(home) if home else Path.home() / ".meshnet") / "checkpoints"


@dataclass
class CheckpointConfig:
    checkpoint_dir: Path = field(default_factory=default_checkpoint_dir)
    max_checkpoints_per_job: int = 5
    max_total_storage_bytes: int = 10 * 1024 ** 3
    retention_period_s: float = 24 * 3600.0
    replicate_to_peers: bool = False
    replication_factor: int = 2


@dataclass
class CheckpointMetadata:
    checkpoint_id: str
    job_id: str
    token_index: int
    created_at: float
    size_bytes: int = 0
    current_layer: int = 0
    model_id: str = ""
    worker_id: str = ""
    data_hash: str = ""


@dataclass
class Checkpoint:
    metadata: CheckpointMetadata
    request: dict
    generated_tokens: List[int]
    config: dict
    kv_handoff: Optional[dict] = None
    rng_state: Optional[bytes] = None

    def payload(self) -> dict:
        d = asdict(self)
        d["metadata"] = dict(d["metadata"])
        d["metadata"]["data_hash"] = ""
        return d

    def compute_hash(self) -> str:
        return hashlib.sha256(cbor2.dumps(self.payload(), canonical=True)).hexdigest()

    def to_bytes(self) -> bytes:
        self.metadata.data_hash = self.compute_hash()
        return cbor2.dumps(asdict(self), canonical=True)

    @classmethod
    def from_bytes(cls, b: bytes, verify: bool = True) -> "Checkpoint":
        d = cbor2.loads(b)
        cp = cls(metadata=CheckpointMetadata(**d["metadata"]), request=d["request"],
                 generated_tokens=list(d["generated_tokens"]), config=d["config"], kv_handoff=d.get("kv_handoff"),
                 rng_state=d.get("rng_state"))
        if verify and cp.metadata.data_hash != cp.compute_hash():
            raise ValueError(f"checkpoint {cp.metadata.checkpoint_id} hash mismatch")
        return cp

    @classmethod
    def new(cls, job_id: str, token_index: int, request: dict, generated: List[int], config: dict,
            kv_handoff: Optional[dict] = None, model_id: str = "", worker_id: str = "") -> "Checkpoint":
        md = CheckpointMetadata(checkpoint_id=str(uuid.uuid4()), job_id=job_id, token_index=token_index,
                                created_at=time.time(), model_id=model_id, worker_id=worker_id)
        return cls(metadata=md, request=request, generated_tokens=list(generated), config=config,
                   kv_handoff=kv_handoff)


class CheckpointManager:
    def __init__(self, config: Optional[CheckpointConfig] = None):
        self.config = config or CheckpointConfig()
        Path(self.config.checkpoint_dir).mkdir(parents=True, exist_ok=True)

    def _job_dir(self, job_id: str) -> Path:
        return Path(self.config.checkpoint_dir) / job_id

    def save(self, cp: Checkpoint) -> Path:
        data = cp.to_bytes()
        cp.metadata.size_bytes = len(data)
        data = cp.to_bytes()
        d = self._job_dir(cp.metadata.job_id)
        d.mkdir(parents=True, exist_ok=True)
        p = d / f"{cp.metadata.checkpoint_id}{CKPT_SUFFIX}"
        tmp = d / f"{cp.metadata.checkpoint_id}{CKPT_SUFFIX}.tmp"
        tmp.write_bytes(data)
        tmp.replace(p)
        self.enforce_retention(cp.metadata.job_id)
        return p

    def list(self, job_id: str) -> List[CheckpointMetadata]:
        d = self._job_dir(job_id)
        out = []
        if d.exists():
            for f in d.glob(f"*{CKPT_SUFFIX}"):
                try:
                    out.append(CheckpointMetadata(**cbor2.loads(f.read_bytes())["metadata"]))
                except Exception:
                    continue
        out.sort(key=lambda m: (m.token_index, m.created_at))
        return out

    def load(self, job_id: str, checkpoint_id: Optional[str] = None) -> Optional[Checkpoint]:
        metas = self.list(job_id)
        if not metas:
            return None
        m = metas[-1] if checkpoint_id is None else next((x for x in metas if x.checkpoint_id == checkpoint_id), None)
        if m is None:
            return None
        return Checkpoint.from_bytes((self._job_dir(job_id) / f"{m.checkpoint_id}{CKPT_SUFFIX}").read_bytes())

    def delete_job(self, job_id: str) -> None:
        shutil.rmtree(self._job_dir(job_id), ignore_errors=True)

    def enforce_retention(self, job_id: Optional[str] = None) -> int:
        """Apply per-job count, age and total-size limits; returns the number of files removed."""
        removed = 0
        root = Path(self.config.checkpoint_dir)
        now = time.time()
        jobs = [job_id] if job_id else [p.name for p in root.iterdir() if p.is_dir()]
        for j in jobs:
            metas = self.list(j)
            for m in metas[:-self.config.max_checkpoints_per_job] if len(metas) > self.config.max_checkpoints_per_job \
                    else []:
                (self._job_dir(j) / f"{m.checkpoint_id}{CKPT_SUFFIX}").unlink(missing_ok=True)
                removed += 1
        files = sorted(root.glob(f"*/*{CKPT_SUFFIX}"), key=lambda f: f.stat().st_mtime)
        for f in files:
            if now - f.stat().st_mtime > self.config.retention_period_s:
                f.unlink(missing_ok=True)
                removed += 1
        files = sorted(root.glob(f"*/*{CKPT_SUFFIX}"), key=lambda f: f.stat().st_mtime)
        total = sum(f.stat().st_size for f in files)
        for f in files:
            if total <= self.config.max_total_storage_bytes:
                break
            total -= f.stat().st_size
            f.unlink(missing_ok=True)
            removed += 1
        return removed
