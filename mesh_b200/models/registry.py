"""Shard registry: which model shards this box holds and where each one is in its lifecycle.

Behaviour of ``agent/src/model/registry.rs:42-310`` and ``agent/src/model/shard.rs:10-225``: a
shard is assigned (``pending``), fetched (``downloading`` with progress, then ``downloaded``
with its path and verified sha256), loaded (``ready`` with the bytes it occupies) and unloaded
again, or marked ``error`` with a message; model descriptions (``ModelInfo``) are registered
beside the shards and the state persists in ``registry.json``.

A B200 box serves one model as a TP group of one process per GPU, each holding one shard, so an
entry is keyed by model and shard position (``<model_id>#<pos>-of-<n>``) rather than by model
alone, records the GPU it is loaded on, and the file is updated under an advisory lock by
read-merge-write, so the ranks of a group can record their own shards concurrently.
"""
from __future__ import annotations

import enum
import fcntl
import json
import os
import threading
import time
from dataclasses import asdict, dataclass, field
from pathlib import Path
from typing import Dict, List, Optional, Tuple

from ..errors import ConfigError, ResourceError
from .artifacts import ShardAssignment


class ShardStatus(str, enum.Enum):
    PENDING = "pending"
    DOWNLOADING = "downloading"
    DOWNLOADED = "downloaded"
    READY = "ready"
    ERROR = "error"


@dataclass
class ModelInfo:
    model_id: str
    name: str = ""
    num_layers: int = 0
    hidden_dim: int = 0
    tensor_parallelism_dim: int = 0
    num_heads: int = 0
    num_kv_heads: int = 0
    vocab_size: int = 0
    total_size_bytes: int = 0
    min_workers: int = 1
    recommended_workers: int = 1
    memory_per_worker_bytes: int = 0
    context_length: int = 0
    format: str = "safetensors"
    shard_urls: List[str] = field(default_factory=list)

    def memory_for_workers(self, n: int) -> int:
        """A worker's share of the weights plus 10% for activations and KV (all of it at n=0)."""
        if n <= 0:
            return self.total_size_bytes
        share = self.total_size_bytes // n
        return share + share // 10

    def columns_per_worker(self, n: int) -> int:
        return self.tensor_parallelism_dim if n <= 0 else self.tensor_parallelism_dim // n

    def can_run_with_workers(self, n: int) -> bool:
        return n >= self.min_workers

    def valid_worker_counts(self) -> List[int]:
        """TP degrees whose shards stay head-aligned: divisors of the KV head count."""
        kv = self.num_kv_heads or 1
        return [n for n in range(1, kv + 1) if kv % n == 0]

    @classmethod
    def from_model_dir(cls, model_dir, gpu_bytes: Optional[int] = None, bytes_per_param: int = 2) -> "ModelInfo":
        """Describe an on-disk mesh model. ``min_workers`` is the smallest head-aligned TP degree
        whose per-GPU share (weights at ``bytes_per_param``, bf16 on the GPU, plus 10%) fits in
        ``gpu_bytes`` of HBM; ``recommended_workers`` the smallest that leaves half of it for KV."""
        from .artifacts import assignment_for, load_model_manifest
        model_dir = Path(model_dir)
        man = load_model_manifest(model_dir)
        shards = sorted(model_dir.glob("shard-*-of-*.manifest.json"))
        if not shards:
            raise ConfigError(f"no shard manifests in {model_dir}")
        total = int(shards[0].name.split("-of-")[1].split(".")[0])
        cfg = _config_of_shard(model_dir, assignment_for(model_dir, man["model_id"], 0, total))
        info = cls(model_id=man["model_id"], name=cfg.name or man["model_id"], num_layers=cfg.num_layers,
                   hidden_dim=cfg.hidden_dim, tensor_parallelism_dim=int(man.get("tensor_parallelism_dim",
                                                                                   cfg.hidden_dim)),
                   num_heads=cfg.num_heads, num_kv_heads=cfg.num_kv_heads, vocab_size=cfg.vocab_size,
                   total_size_bytes=int(cfg.param_count() * bytes_per_param), context_length=int(man.get("context_length", 0)),
                   shard_urls=[f"file://{model_dir / p.name.replace('.manifest.json', '.safetensors')}"
                               for p in shards])
        counts = info.valid_worker_counts()
        if gpu_bytes:
            fits = [n for n in counts if info.memory_for_workers(n) <= gpu_bytes]
            roomy = [n for n in counts if info.memory_for_workers(n) <= gpu_bytes // 2]
            if not fits:
                raise ResourceError(f"{info.model_id} does not fit {len(counts) and counts[-1]} GPUs of "
                                    f"{gpu_bytes} bytes")
            info.min_workers = fits[0]
            info.recommended_workers = roomy[0] if roomy else counts[-1]
        info.memory_per_worker_bytes = info.memory_for_workers(info.recommended_workers)
        return info


def _config_of_shard(model_dir: Path, a: ShardAssignment):
    from safetensors import safe_open
    from ..config import ModelConfig
    path = model_dir / f"shard-{a.worker_position}-of-{a.total_workers}.safetensors"
    with safe_open(str(path), framework="np") as f:
        return ModelConfig.from_metadata(f.metadata() or {})


def assignment_by_columns(model_id: str, position: int, total: int, total_columns: int) -> ShardAssignment:
    """Even column split; the last worker takes the remainder."""
    per = total_columns // total
    end = total_columns if position == total - 1 else (position + 1) * per
    return ShardAssignment(model_id, position, total, position * per, end)


@dataclass
class ShardInfo:
    assignment: ShardAssignment
    status: ShardStatus = ShardStatus.PENDING
    error: Optional[str] = None
    is_loaded: bool = False
    memory_bytes: int = 0
    device: Optional[str] = None
    file_path: Optional[str] = None
    file_hash: Optional[str] = None
    download_progress: float = 0.0
    last_verified: Optional[int] = None

    @property
    def key(self) -> str:
        a = self.assignment
        return shard_key(a.model_id, a.worker_position, a.total_workers)

    def num_columns(self) -> int:
        return self.assignment.column_end - self.assignment.column_start

    def contains_column(self, c: int) -> bool:
        return self.assignment.column_start <= c < self.assignment.column_end

    def to_json(self) -> dict:
        d = asdict(self)
        d["status"] = self.status.value
        return d

    @classmethod
    def from_json(cls, d: dict) -> "ShardInfo":
        d = dict(d)
        d["assignment"] = ShardAssignment(**d["assignment"])
        d["status"] = ShardStatus(d["status"])
        return cls(**d)


def shard_key(model_id: str, position: int, total: int) -> str:
    return f"{model_id}#{position}-of-{total}"


def default_registry_dir() -> Path:
    home = os.environ.get("MESHNET_HOME")
    return (Path(home) if home else Path.home() / ".meshnet") / "shards"


class ShardRegistry:
    """The shards and model descriptions of this box, persisted in ``<dir>/registry.json``."""

    def __init__(self, storage_dir=None):
        self.dir = Path(storage_dir) if storage_dir else default_registry_dir()
        self.dir.mkdir(parents=True, exist_ok=True)
        self.file = self.dir / "registry.json"
        self._lock = threading.Lock()
        self.shards: Dict[str, ShardInfo] = {}
        self.models: Dict[str, ModelInfo] = {}
        self._dirty: set = set()
        self._removed: set = set()
        self.load()

    # ------------------------------------------------------------------ persistence
    def _read_file(self) -> Tuple[Dict[str, ShardInfo], Dict[str, ModelInfo]]:
        if not self.file.exists():
            return {}, {}
        try:
            d = json.loads(self.file.read_text() or "{}")
        except json.JSONDecodeError as e:
            raise ConfigError(f"corrupt shard registry {self.file}: {e}") from e
        return ({k: ShardInfo.from_json(v) for k, v in d.get("shards", {}).items()},
                {k: ModelInfo(**v) for k, v in d.get("models", {}).items()})

    def load(self) -> None:
        with self._lock, open(self.dir / "registry.lock", "a") as lk:
            fcntl.flock(lk, fcntl.LOCK_SH)
            self.shards, self.models = self._read_file()
            self._dirty.clear()
            self._removed.clear()

    def save(self) -> None:
        """Merge this process's changed entries into the file (other processes' entries are
        kept) and write it atomically."""
        with self._lock, open(self.dir / "registry.lock", "a") as lk:
            fcntl.flock(lk, fcntl.LOCK_EX)
            shards, models = self._read_file()
            for k in self._dirty:
                if k in self.shards:
                    shards[k] = self.shards[k]
            for k in self._removed:
                shards.pop(k, None)
            models.update(self.models)
            tmp = self.file.with_suffix(f".tmp{os.getpid()}")
            tmp.write_text(json.dumps({"shards": {k: v.to_json() for k, v in sorted(shards.items())},
                                       "models": {k: asdict(v) for k, v in sorted(models.items())}}, indent=2))
            os.replace(tmp, self.file)
            self.shards = {**shards, **{k: self.shards[k] for k in self._dirty if k in self.shards}}
            self.models = models
            self._dirty.clear()
            self._removed.clear()

    # ------------------------------------------------------------------ models
    def register_model(self, info: ModelInfo) -> None:
        self.models[info.model_id] = info
        self.save()

    def get_model(self, model_id: str) -> Optional[ModelInfo]:
        return self.models.get(model_id)

    def list_models(self) -> List[ModelInfo]:
        return list(self.models.values())

    # ------------------------------------------------------------------ shards
    def _get(self, key: str) -> ShardInfo:
        s = self.shards.get(key)
        if s is None:
            raise ConfigError(f"shard {key} is not assigned to this device")
        return s

    def _touch(self, s: ShardInfo) -> ShardInfo:
        self._dirty.add(s.key)
        self._removed.discard(s.key)
        self.save()
        return s

    def assign_shard(self, a: ShardAssignment) -> ShardInfo:
        """Assign (or re-assign) a shard; a re-assignment with another column range starts over."""
        if not (0 <= a.worker_position < a.total_workers) or a.column_end <= a.column_start:
            raise ConfigError(f"invalid shard assignment {a}")
        k = shard_key(a.model_id, a.worker_position, a.total_workers)
        cur = self.shards.get(k)
        if cur is not None and cur.assignment == a:
            return cur
        s = ShardInfo(assignment=a)
        self.shards[k] = s
        return self._touch(s)

    def get_shard(self, key: str) -> Optional[ShardInfo]:
        return self.shards.get(key)

    def status(self, key: str) -> Optional[ShardStatus]:
        s = self.shards.get(key)
        return s.status if s else None

    def update_status(self, key: str, status: ShardStatus, error: Optional[str] = None) -> ShardInfo:
        s = self._get(key)
        s.status = ShardStatus(status)
        s.error = error if s.status == ShardStatus.ERROR else None
        return self._touch(s)

    def update_download_progress(self, key: str, progress: float) -> ShardInfo:
        s = self._get(key)
        s.status = ShardStatus.DOWNLOADING
        s.download_progress = min(1.0, max(0.0, float(progress)))
        return self._touch(s)

    def mark_downloaded(self, key: str, path, file_hash: str) -> ShardInfo:
        s = self._get(key)
        s.status, s.file_path, s.file_hash = ShardStatus.DOWNLOADED, str(path), file_hash
        s.download_progress, s.last_verified = 1.0, int(time.time())
        return self._touch(s)

    def mark_loaded(self, key: str, memory_bytes: int, device: Optional[str] = None) -> ShardInfo:
        s = self._get(key)
        if s.status not in (ShardStatus.DOWNLOADED, ShardStatus.READY):
            raise ConfigError(f"shard {key} is {s.status.value}; it must be downloaded before it loads")
        s.status, s.is_loaded, s.memory_bytes, s.device = ShardStatus.READY, True, int(memory_bytes), device
        return self._touch(s)

    def mark_unloaded(self, key: str) -> ShardInfo:
        s = self._get(key)
        if s.is_loaded:
            s.status = ShardStatus.DOWNLOADED
        s.is_loaded, s.memory_bytes, s.device = False, 0, None
        return self._touch(s)

    def mark_error(self, key: str, message: str) -> ShardInfo:
        return self.update_status(key, ShardStatus.ERROR, message)

    def remove_shard(self, key: str) -> None:
        self._get(key)
        del self.shards[key]
        self._dirty.discard(key)
        self._removed.add(key)
        self.save()

    def list_shards(self) -> List[ShardInfo]:
        return [self.shards[k] for k in sorted(self.shards)]

    def ready_shards(self) -> List[ShardInfo]:
        return [s for s in self.list_shards() if s.status == ShardStatus.READY]

    def total_memory_usage(self) -> int:
        return sum(s.memory_bytes for s in self.shards.values() if s.is_loaded)

    def is_ready(self, key: str) -> bool:
        s = self.shards.get(key)
        return bool(s and s.status == ShardStatus.READY)

    def shard_path(self, model_id: str) -> Path:
        return self.dir / model_id

    def summary(self) -> dict:
        return {"shards": {k: v.to_json() for k, v in sorted(self.shards.items())},
                "models": {k: asdict(v) for k, v in sorted(self.models.items())},
                "total_memory_usage": self.total_memory_usage()}


def record_shard_load(registry: Optional["ShardRegistry"], model_dir, a: ShardAssignment, memory_bytes: int,
                      device: str) -> Optional[str]:
    """After ``artifacts.load_shard`` verified a shard and its weights are on ``device``: record it
    downloaded (path, hash from its manifest) and ready. Returns the entry's key."""
    if registry is None:
        return None
    man = json.loads((Path(model_dir) / f"shard-{a.worker_position}-of-{a.total_workers}.manifest.json").read_text())
    k = registry.assign_shard(a).key
    registry.mark_downloaded(k, Path(model_dir) / f"shard-{a.worker_position}-of-{a.total_workers}.safetensors",
                             man["expected_sha256"])
    registry.mark_loaded(k, memory_bytes, device)
    return k
