"""Resource manager: the memory a device commits to the mesh, with a lock cooldown.

Behaviour of ``agent/src/resource_manager.rs:1-620``: a user allocation gets a 7% safety margin,
locking it starts a cooldown (24 h by default) before unlock is allowed (``CooldownActive``
reports the hours left, rounded up), the commitment survives restarts (written atomically to
``resource_lock.toml``) and is re-pinned on load, and an unpinnable commitment stays a commitment.

On a B200 box the memory that serves is HBM, so a commitment names its pool:

* ``hbm`` (the default when GPUs are present): bytes per GPU. Nothing is pinned on the host;
  the lock checks that every GPU has that much free at lock time, and the serving runtime sizes
  its KV page pool from the commitment (``kv_pages_for``) instead of from whatever is free.
* ``host``: host RAM, pinned with ``mlock`` on an anonymous mapping held for the manager's life
  (the host staging that CPU ranks and checkpoint uploads use).

Sizes parse as the reference's strings do (``7GB`` = 7e9 bytes, ``7GiB`` = 7·2^30, plain
integers are bytes); single-letter binary suffixes (``16G``) are also accepted.
"""
from __future__ import annotations

import ctypes
import mmap
import os
import time
from dataclasses import asdict, dataclass
from pathlib import Path
from typing import List, Optional

from ..errors import ConfigError, CooldownActive, ResourceError

SAFETY_MARGIN = 1.07
DEFAULT_COOLDOWN_HOURS = 24


def parse_memory_string(s: str) -> int:
    t = str(s).strip().upper().replace(" ", "")
    units = (("TIB", 1 << 40), ("GIB", 1 << 30), ("MIB", 1 << 20), ("KIB", 1 << 10),
             ("TB", 10 ** 12), ("GB", 10 ** 9), ("MB", 10 ** 6), ("KB", 10 ** 3),
             ("T", 1 << 40), ("G", 1 << 30), ("M", 1 << 20), ("K", 1 << 10))
    for suf, mult in units:
        if t.endswith(suf):
            try:
                v = float(t[:-len(suf)])
            except ValueError:
                break
            if v < 0:
                break
            return int(v * mult)
    else:
        if t.isdigit():
            return int(t)
    raise ConfigError(f"invalid memory size {s!r}: use e.g. '7GB', '7GiB', '512MB' or a byte count")


def format_bytes(n: int) -> str:
    for unit, div in (("GB", 10 ** 9), ("MB", 10 ** 6), ("KB", 10 ** 3)):
        if n >= div:
            return f"{n / div:.1f} {unit}"
    return f"{n} bytes"


def host_total_memory() -> int:
    return os.sysconf("SC_PAGE_SIZE") * os.sysconf("SC_PHYS_PAGES")


def gpu_memory() -> List[int]:
    """Total HBM of each visible GPU (empty without CUDA)."""
    try:
        import torch
        if torch.cuda.is_available():
            return [torch.cuda.get_device_properties(i).total_memory for i in range(torch.cuda.device_count())]
    except Exception:
        pass
    return []


def kv_pages_for(committed_bytes: int, weight_bytes: int, page_bytes: int, workspace_bytes: int = 2 << 30) -> int:
    """KV pages one GPU can hold within its commitment after its weights and a workspace
    reserve (activations, graphs' buffers, collective workspaces)."""
    free = committed_bytes - weight_bytes - workspace_bytes
    if free < page_bytes:
        raise ResourceError(f"commitment {format_bytes(committed_bytes)} leaves no room for KV pages after "
                            f"{format_bytes(weight_bytes)} of weights and {format_bytes(workspace_bytes)} of workspace")
    return int(free // page_bytes)


@dataclass
class ResourceLockConfig:
    pool: str = "host"
    user_allocated: int = 0
    locked_memory: int = 0
    lock_timestamp: Optional[int] = None
    cooldown_hours: int = DEFAULT_COOLDOWN_HOURS


class _PinnedRegion:
    """An anonymous mapping whose pages are locked in RAM until ``release``."""

    def __init__(self, size: int):
        self.size = size
        self.map = mmap.mmap(-1, size)
        self._cbuf = (ctypes.c_char * size).from_buffer(self.map)
        libc = ctypes.CDLL(None, use_errno=True)
        self._munlock = libc.munlock
        if libc.mlock(ctypes.c_void_p(ctypes.addressof(self._cbuf)), ctypes.c_size_t(size)) != 0:
            err = ctypes.get_errno()
            self._drop()
            raise ResourceError(f"mlock of {format_bytes(size)} failed: {os.strerror(err)}")

    def _drop(self):
        del self._cbuf
        self.map.close()

    def release(self):
        self._munlock(ctypes.c_void_p(ctypes.addressof(self._cbuf)), ctypes.c_size_t(self.size))
        self._drop()


class ResourceManager:
    def __init__(self, config_path, pool: Optional[str] = None, host_total: Optional[int] = None,
                 gpu_totals: Optional[List[int]] = None, gpu_free=None):
        self.config_path = Path(config_path)
        self.gpu_totals = gpu_memory() if gpu_totals is None else list(gpu_totals)
        self.host_total = host_total_memory() if host_total is None else int(host_total)
        self._gpu_free = gpu_free  # callable -> [free bytes per GPU]; torch's mem_get_info by default
        self.cfg = ResourceLockConfig(pool=pool or ("hbm" if self.gpu_totals else "host"))
        self._pinned: Optional[_PinnedRegion] = None
        self.load_config()
        if pool is not None and not self.is_locked:
            self.cfg.pool = pool

    # ------------------------------------------------------------------ state
    @property
    def pool(self) -> str:
        return self.cfg.pool

    @property
    def total_memory(self) -> int:
        """Per-GPU HBM (the smallest GPU) for ``hbm``, host RAM for ``host``."""
        if self.pool == "hbm":
            if not self.gpu_totals:
                raise ResourceError("no GPU visible for an hbm commitment")
            return min(self.gpu_totals)
        return self.host_total

    @property
    def is_locked(self) -> bool:
        return self.cfg.lock_timestamp is not None

    @property
    def is_pinned(self) -> bool:
        return self._pinned is not None

    def time_until_unlock(self, now: Optional[float] = None) -> float:
        if not self.is_locked:
            return 0.0
        left = self.cfg.lock_timestamp + self.cfg.cooldown_hours * 3600 - (time.time() if now is None else now)
        return max(0.0, left)

    def status(self) -> dict:
        d = asdict(self.cfg)
        d.update(locked=self.is_locked, pinned=self.is_pinned, total_memory=self.total_memory,
                 seconds_until_unlock=self.time_until_unlock(), gpus=len(self.gpu_totals),
                 locked_human=format_bytes(self.cfg.locked_memory))
        return d

    # ------------------------------------------------------------------ actions
    def set_allocation(self, nbytes: int, cooldown_hours: Optional[int] = None) -> None:
        if self.is_locked:
            raise ResourceError("memory is locked; unlock it before changing the allocation")
        nbytes = int(nbytes)
        total = self.total_memory
        if nbytes <= 0 or nbytes > total:
            raise ResourceError(f"requested {format_bytes(nbytes)} is outside (0, {format_bytes(total)}]")
        buffered = int(nbytes * SAFETY_MARGIN)
        if buffered > total:
            raise ResourceError(f"allocation with its 7% margin ({format_bytes(buffered)}) exceeds "
                                f"{format_bytes(total)}")
        self.cfg.user_allocated, self.cfg.locked_memory = nbytes, buffered
        if cooldown_hours is not None:
            self.cfg.cooldown_hours = int(cooldown_hours)

    def lock(self, pin: bool = True) -> None:
        """Start the commitment. ``pin=False`` records it without pinning host memory now (a CLI
        process that exits at once); the long-lived runtime pins it when it loads the config."""
        if self.is_locked:
            raise ResourceError("memory already locked")
        if self.cfg.locked_memory == 0:
            raise ResourceError("no allocation set; call set_allocation first")
        if pin or self.pool == "hbm":
            self._reserve()
        self.cfg.lock_timestamp = int(time.time())
        self.save_config()

    def unlock(self, now: Optional[float] = None) -> None:
        if not self.is_locked:
            raise ResourceError("memory is not locked")
        left = self.time_until_unlock(now)
        if left > 0:
            raise CooldownActive(-(-int(left) // 3600))
        if self._pinned is not None:
            self._pinned.release()
            self._pinned = None
        self.cfg.lock_timestamp = None
        self.save_config()

    def _reserve(self) -> None:
        if self.pool == "host":
            self._pinned = _PinnedRegion(self.cfg.locked_memory)
            return
        free = self._gpu_free() if self._gpu_free else self._torch_free()
        short = [i for i, f in enumerate(free) if f < self.cfg.locked_memory]
        if short:
            raise ResourceError(f"GPU(s) {short} have less than {format_bytes(self.cfg.locked_memory)} free")

    @staticmethod
    def _torch_free() -> List[int]:
        import torch
        out = []
        for i in range(torch.cuda.device_count()):
            with torch.cuda.device(i):
                out.append(torch.cuda.mem_get_info()[0])
        return out

    # ------------------------------------------------------------------ persistence
    def save_config(self) -> None:
        self.config_path.parent.mkdir(parents=True, exist_ok=True)
        lines = [f"pool = \"{self.cfg.pool}\"", f"user_allocated = {self.cfg.user_allocated}",
                 f"locked_memory = {self.cfg.locked_memory}", f"cooldown_hours = {self.cfg.cooldown_hours}"]
        if self.cfg.lock_timestamp is not None:
            lines.append(f"lock_timestamp = {self.cfg.lock_timestamp}")
        tmp = self.config_path.with_suffix(".tmp")
        tmp.write_text("\n".join(lines) + "\n")
        os.replace(tmp, self.config_path)  # atomic on POSIX

    def load_config(self) -> None:
        if not self.config_path.exists():
            return
        import tomllib
        try:
            d = tomllib.loads(self.config_path.read_text())
        except Exception as e:
            raise ConfigError(f"invalid resource lock file {self.config_path}: {e}") from e
        self.cfg = ResourceLockConfig(**{k: d[k] for k in asdict(ResourceLockConfig()) if k in d})
        if self.is_locked and self.pool == "host" and self.cfg.locked_memory > 0:
            try:  # re-pin after a restart; a failure leaves the commitment standing, unpinned
                self._pinned = _PinnedRegion(self.cfg.locked_memory)
            except ResourceError:
                self._pinned = None

    def close(self) -> None:
        if self._pinned is not None:
            self._pinned.release()
            self._pinned = None
