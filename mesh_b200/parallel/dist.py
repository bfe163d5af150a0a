"""Process-group bootstrap: one process per GPU, NCCL for GPU ranks, gloo for CPU ranks.

Rendezvous uses the standard torchrun environment (RANK, WORLD_SIZE, LOCAL_RANK, MASTER_ADDR,
MASTER_PORT). The process-group timeout is short by default so a lost rank surfaces as an error
instead of a hang (the reference's 30 s all-reduce timeout, coordinator.rs:117).
"""
from __future__ import annotations

import datetime
import os
from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist


@dataclass
class DistInfo:
    rank: int = 0
    world: int = 1
    local_rank: int = 0
    device: torch.device = torch.device("cpu")
    backend: str = "none"

    @property
    def is_main(self) -> bool:
        return self.rank == 0


_INFO: Optional[DistInfo] = None


def init(backend: Optional[str] = None, timeout_s: float = 60.0, device: Optional[str] = None) -> DistInfo:
    """Initialise (or return) the process group from torchrun env vars; single-process if absent."""
    global _INFO
    if _INFO is not None:
        return _INFO
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    use_cuda = torch.cuda.is_available() and device != "cpu"
    if use_cuda:
        torch.cuda.set_device(local % torch.cuda.device_count())
        dev = torch.device("cuda", torch.cuda.current_device())
    else:
        dev = torch.device("cpu")
    be = "none"
    if world > 1:
        be = backend or ("nccl" if use_cuda else "gloo")
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        kw = dict(backend=be, rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))
        if be == "nccl":
            kw["device_id"] = dev
        if not dist.is_initialized():
            dist.init_process_group(**kw)
    _INFO = DistInfo(rank=rank, world=world, local_rank=local, device=dev, backend=be)
    return _INFO


def info() -> DistInfo:
    return _INFO if _INFO is not None else DistInfo()


def shutdown():
    global _INFO
    if dist.is_available() and dist.is_initialized():
        try:
            dist.barrier()
        except Exception:
            pass
        dist.destroy_process_group()
    _INFO = None
