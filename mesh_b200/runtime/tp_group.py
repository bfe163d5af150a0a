"""Tensor-parallel worker group on one box: rank 0 drives the serving engine of the whole group.

The reference runs one ``mesh device runtime`` per ring member; the members of a TP ring execute
the same forward in lock step and meet in their TCP ring all-reduce (``agent/src/main.rs:3629-4787``,
``agent/src/inference/forward_pass.rs:1946-2025``). On a B200 box the members are one process per
GPU. Rank 0 (the leader) runs the worker loop and the coordinator; every call it makes on its
backend (prefill, decode, release, KV export / import) is first broadcast to the followers, which
make the same call on their own engine. Every engine decision depends only on those calls and on
the engine's own state, so all ranks launch the same kernels and collectives in the same order.

Control messages go over a gloo process group (host memory), apart from the NCCL group and the
peer-memory kernels, so they never queue behind GPU work. A follower that dies makes the leader's
next broadcast fail (connection closed or the group's timeout), which ends the leader's call with
an exception the worker loop reports (the lease is released and the sessions retried elsewhere).

KV checkpoints of a TP group hold one part per rank (each rank owns its KV heads); they are
imported by a group of the same TP degree.
"""
from __future__ import annotations

import datetime
import os
from dataclasses import dataclass
from pathlib import Path
from typing import Callable, List, Optional

import cbor2

TP_PARTS_ENCODING = "tp_parts_v1"
_STOP = "__stop__"


class TPGroupBackend:
    """Leader-side backend: broadcasts each call to the followers, then runs it locally."""

    def __init__(self, backend, group, world: int):
        import torch.distributed as dist
        self.b = backend
        self.group = group
        self.world = world
        self.dist = dist
        self.provider = getattr(backend, "provider", "cuda")
        self.class_key = getattr(backend, "class_key", 1)
        self.calls = 0

    # ------------------------------------------------------------------ plumbing
    def _announce(self, name: str, *args):
        self.dist.broadcast_object_list([(name, args)], src=0, group=self.group)
        self.calls += 1

    def _call(self, name: str, *args):
        self._announce(name, *args)
        return getattr(self.b, name)(*args)

    def stop(self):
        """Release the followers (they return from ``follow``)."""
        self._announce(_STOP)

    # ------------------------------------------------------------------ backend interface
    def token_ceiling(self, n: int) -> int:
        return self.b.token_ceiling(n)

    def prefill(self, h, prompt, temperature, top_p, seed_base):
        return self._call("prefill", h, prompt, temperature, top_p, seed_base)

    def decode(self, items):
        return self._call("decode", items)

    def release(self, h):
        return self._call("release", h)

    def drain_counters(self):
        # local bookkeeping only: nothing is announced, the followers keep their own counters
        return self.b.drain_counters() if hasattr(self.b, "drain_counters") else {}

    def kv_bytes(self, h) -> int:
        # every rank holds the same number of pages for a session (its own KV heads)
        return self.b.kv_bytes(h) * self.world

    def export_kv(self, h) -> bytes:
        self._announce("export_kv", h)
        mine = self.b.export_kv(h)
        parts: List[Optional[bytes]] = [None] * self.world
        self.dist.gather_object(mine, parts, dst=0, group=self.group)
        return cbor2.dumps({"encoding": TP_PARTS_ENCODING, "world": self.world, "parts": parts})

    def import_kv(self, h, payload: bytes, prompt, generated):
        d = cbor2.loads(payload)
        if not isinstance(d, dict) or d.get("encoding") != TP_PARTS_ENCODING:
            raise ValueError("a TP group imports KV checkpoints written by a TP group (tp_parts_v1)")
        if d["world"] != self.world:
            raise ValueError(f"KV checkpoint has {d['world']} rank parts; this group has {self.world} ranks")
        self._announce("import_kv", h, prompt, generated)
        out = [None]
        self.dist.scatter_object_list(out, list(d["parts"]), src=0, group=self.group)
        return self.b.import_kv(h, out[0], prompt, generated)


def follow(backend, group) -> int:
    """Follower loop: make every call the leader announces on the local backend, until stopped.
    Returns the number of calls made."""
    import torch.distributed as dist
    n = 0
    while True:
        box = [None]
        dist.broadcast_object_list(box, src=0, group=group)
        name, args = box[0]
        if name == _STOP:
            return n
        n += 1
        if name == "export_kv":
            mine = backend.export_kv(*args)
            dist.gather_object(mine, None, dst=0, group=group)
        elif name == "import_kv":
            h, prompt, generated = args
            part = [None]
            dist.scatter_object_list(part, None, src=0, group=group)
            backend.import_kv(h, part[0], prompt, generated)
        else:
            getattr(backend, name)(*args)


# ---------------------------------------------------------------------------------- group launch
@dataclass
class GroupSpec:
    """What every rank of a group builds: the model (an on-disk model directory with shards for
    ``world`` ranks, or a preset with synthetic weights), the engine sizes and the device offset."""
    world: int
    model_dir: Optional[str] = None
    preset: Optional[str] = None
    seed: int = 0
    max_seq_len: int = 4096
    num_pages: int = 4096
    max_batch: int = 64
    max_tokens: int = 8192
    use_cuda_graphs: bool = True
    first_device: int = 0
    timeout_s: float = 120.0
    registry_dir: Optional[str] = None   # shard registry each rank records its shard in
    hbm_commit_bytes: int = 0            # per-GPU commitment: sizes the KV pool when set


def build_rank_backend(spec: GroupSpec, rank: int, group=None):
    """This rank's engine on ``cuda:first_device+rank`` with its weights shard, wrapped as a
    ``GpuBackend``. Weights come from ``shard-<rank>-of-<world>`` of the model directory (hash and
    shapes checked) or are the preset's synthetic weights."""
    import torch
    from ..config import EngineConfig, get_preset
    from ..engine.backend import GpuBackend
    from ..engine.serving import Engine
    from ..models.llama import KVPool, LlamaRunner
    dev = torch.device("cuda", spec.first_device + rank)
    torch.cuda.set_device(dev)
    base = torch.cuda.memory_allocated(dev)
    registry = shard = None
    if spec.model_dir:
        from ..models.artifacts import assignment_for, load_model_manifest, load_shard, shard_to_device_weights
        man = load_model_manifest(Path(spec.model_dir))
        a = assignment_for(Path(spec.model_dir), man["model_id"], rank, spec.world)
        if spec.registry_dir:
            from ..models.registry import ShardRegistry
            registry = ShardRegistry(spec.registry_dir)
            shard = registry.assign_shard(a).key
        try:
            cfg, tensors = load_shard(Path(spec.model_dir), a)
        except Exception as e:
            if registry is not None:
                registry.mark_error(shard, str(e))
            raise
        w = shard_to_device_weights(cfg, tensors, rank, spec.world, device=dev)
        del tensors
    else:
        from ..models.weights import synthetic_device_weights
        cfg = get_preset(spec.preset or "small")
        w = synthetic_device_weights(cfg, rank, spec.world, seed=spec.seed, device=dev)
    weight_bytes = torch.cuda.memory_allocated(dev) - base
    if registry is not None:
        from ..models.registry import record_shard_load
        record_shard_load(registry, spec.model_dir, a, weight_bytes, str(dev))
    ecfg = EngineConfig(max_seq_len=spec.max_seq_len, use_cuda_graphs=spec.use_cuda_graphs, tp=spec.world)
    num_pages = spec.num_pages
    if spec.hbm_commit_bytes:
        from .resources import kv_pages_for
        num_pages = kv_pages_for(spec.hbm_commit_bytes, weight_bytes,
                                 KVPool.bytes_per_page(cfg, w.layout.local_kv_heads, ecfg.page_size))
    kv = KVPool(cfg, w.layout.local_kv_heads, num_pages, ecfg.page_size, dev)
    runner = LlamaRunner(w, ecfg, kv, dev, group=group, max_tokens=spec.max_tokens)
    backend = GpuBackend(Engine(runner, ecfg, max_batch=spec.max_batch))
    backend.registry, backend.shard_key = registry, shard
    return backend, cfg, ecfg


def _rank_main(rank: int, spec: GroupSpec, init_file: str, leader: Callable, result_path: Optional[str],
               spmd: bool = False):
    import torch
    import torch.distributed as dist
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    torch.cuda.set_device(spec.first_device + rank)
    dist.init_process_group("nccl", init_method=f"file://{init_file}", rank=rank, world_size=spec.world,
                            timeout=datetime.timedelta(seconds=spec.timeout_s),
                            device_id=torch.device("cuda", spec.first_device + rank))
    ctl = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=spec.timeout_s))
    try:
        backend, cfg, ecfg = build_rank_backend(spec, rank, group=dist.group.WORLD if spec.world > 1 else None)
        if spmd:
            # every rank runs the leader's program on its own backend (it must be deterministic)
            out = leader(backend, cfg, ecfg)
            if rank == 0 and result_path:
                with open(result_path, "wb") as f:
                    f.write(cbor2.dumps(out))
        elif rank == 0:
            tb = TPGroupBackend(backend, ctl, spec.world)
            try:
                out = leader(tb, cfg, ecfg)
            finally:
                tb.stop()
            if result_path:
                with open(result_path, "wb") as f:
                    f.write(cbor2.dumps(out))
        else:
            follow(backend, ctl)
        torch.cuda.synchronize()
        backend.eng.close()
        if getattr(backend, "registry", None) is not None:
            backend.registry.mark_unloaded(backend.shard_key)
    finally:
        dist.destroy_process_group()


def run_group(spec: GroupSpec, leader: Callable, workdir: str, spmd: bool = False):
    """Start one process per GPU, run ``leader(backend, model_config, engine_config)`` on rank 0 with
    the group backend, and return its (CBOR-serialisable) result once every rank has exited.
    ``spmd=True`` instead runs ``leader`` on every rank with that rank's own backend (each rank makes
    the same calls itself, as the benchmark does); a deterministic program gives the same result."""
    import torch.multiprocessing as mp
    init_file = os.path.join(workdir, "tp_group_store")
    result_path = os.path.join(workdir, "tp_group_result.cbor")
    mp.spawn(_rank_main, args=(spec, init_file, leader, result_path, spmd), nprocs=spec.world, join=True)
    with open(result_path, "rb") as f:
        return cbor2.loads(f.read())
