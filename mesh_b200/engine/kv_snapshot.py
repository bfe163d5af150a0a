"""KV snapshots: export a session's paged K/V to a host blob and import it into another pool.

The reference serialises a host ``KVCache`` (fp32 per layer) as CBOR inside checkpoints and live
transfers (``agent/src/inference/kv_cache.rs:102-187``, ``:880``; window limited to the last 1024
tokens, ``coordinator.rs:90-91``). Here the device pool is paged bf16, so a snapshot gathers the
session's pages (``[layers, tokens, kv_heads, head_dim]`` bf16) into one host buffer and records
the sequence state; import allocates pages and scatters the rows back. Between two ranks of one box
the same gathered tensor can travel GPU to GPU over NVLink (``send_kv`` / ``recv_kv``).
"""
from __future__ import annotations

from dataclasses import asdict, dataclass
from typing import List, Optional

import cbor2
import numpy as np
import torch

ENCODING = "b200_paged_bf16_v1"


@dataclass
class KVSequenceState:
    base_position: int
    next_position: int
    seq_len: int
    window: Optional[int] = None


@dataclass
class KVCacheSnapshot:
    model_id: str
    num_layers: int
    kv_heads: int
    head_dim: int
    sequence: KVSequenceState
    k: bytes
    v: bytes
    encoding: str = ENCODING

    def to_bytes(self) -> bytes:
        d = asdict(self)
        return cbor2.dumps(d)

    @classmethod
    def from_bytes(cls, b: bytes) -> "KVCacheSnapshot":
        d = cbor2.loads(b)
        if d.get("encoding") != ENCODING:
            raise ValueError(f"unsupported KV snapshot encoding {d.get('encoding')!r}")
        d["sequence"] = KVSequenceState(**d["sequence"])
        return cls(**d)

    def tensors(self):
        shape = (self.num_layers, self.sequence.seq_len, self.kv_heads, self.head_dim)
        k = torch.frombuffer(bytearray(self.k), dtype=torch.bfloat16).view(shape)
        v = torch.frombuffer(bytearray(self.v), dtype=torch.bfloat16).view(shape)
        return k, v


def gather_pages(pool_k: torch.Tensor, pool_v: torch.Tensor, pages: List[int], seq_len: int):
    """[layers, pages, hkv, ps, D] pools -> contiguous [layers, seq_len, hkv, D] K and V on the pool's device."""
    idx = torch.tensor(pages, dtype=torch.long, device=pool_k.device)
    L, _, hkv, ps, D = pool_k.shape
    k = pool_k.index_select(1, idx).permute(0, 1, 3, 2, 4).reshape(L, -1, hkv, D)[:, :seq_len]
    v = pool_v.index_select(1, idx).permute(0, 1, 3, 2, 4).reshape(L, -1, hkv, D)[:, :seq_len]
    return k.contiguous(), v.contiguous()


def scatter_pages(pool_k: torch.Tensor, pool_v: torch.Tensor, pages: List[int], k: torch.Tensor, v: torch.Tensor):
    L, _, hkv, ps, D = pool_k.shape
    T = k.shape[1]
    n = (T + ps - 1) // ps
    if len(pages) < n:
        raise ValueError(f"{len(pages)} pages cannot hold {T} tokens")
    pad = n * ps - T
    if pad:
        z = torch.zeros(L, pad, hkv, D, dtype=k.dtype, device=k.device)
        k, v = torch.cat([k, z], 1), torch.cat([v, z], 1)
    idx = torch.tensor(pages[:n], dtype=torch.long, device=pool_k.device)
    kp = k.to(pool_k.device).view(L, n, ps, hkv, D).permute(0, 1, 3, 2, 4)
    vp = v.to(pool_v.device).view(L, n, ps, hkv, D).permute(0, 1, 3, 2, 4)
    pool_k.index_copy_(1, idx, kp.contiguous())
    pool_v.index_copy_(1, idx, vp.contiguous())


def export_snapshot(pool_k, pool_v, pages: List[int], seq: KVSequenceState, model_id: str,
                    max_tokens: Optional[int] = None) -> KVCacheSnapshot:
    k, v = gather_pages(pool_k, pool_v, pages, seq.seq_len)
    if max_tokens is not None and seq.seq_len > max_tokens:
        raise ValueError("snapshot window smaller than the sequence; paged export keeps the whole context")
    L, T, hkv, D = k.shape
    kb = k.cpu().view(torch.int16).numpy().tobytes()
    vb = v.cpu().view(torch.int16).numpy().tobytes()
    return KVCacheSnapshot(model_id=model_id, num_layers=L, kv_heads=hkv, head_dim=D, sequence=seq, k=kb, v=vb)


def import_snapshot(pool_k, pool_v, alloc, snap: KVCacheSnapshot) -> List[int]:
    L, _, hkv, ps, D = pool_k.shape
    if (snap.num_layers, snap.kv_heads, snap.head_dim) != (L, hkv, D):
        raise ValueError("KV snapshot geometry does not match this pool")
    n = (snap.sequence.seq_len + ps - 1) // ps
    pages = alloc.alloc(n)
    if pages is None:
        raise RuntimeError("KV page pool exhausted during import")
    k, v = snap.tensors()
    scatter_pages(pool_k, pool_v, list(pages), k, v)
    return list(pages)


def send_kv(pool_k, pool_v, pages: List[int], seq_len: int, dst: int, group=None):
    """GPU-to-GPU handoff of a session's K/V to rank ``dst`` (NCCL point-to-point over NVLink)."""
    import torch.distributed as dist
    k, v = gather_pages(pool_k, pool_v, pages, seq_len)
    dist.send(torch.tensor([seq_len], device=pool_k.device), dst, group=group)
    dist.send(torch.stack([k, v]), dst, group=group)


def recv_kv(pool_k, pool_v, alloc, src: int, group=None) -> List[int]:
    import torch.distributed as dist
    L, _, hkv, ps, D = pool_k.shape
    t = torch.zeros(1, dtype=torch.long, device=pool_k.device)
    dist.recv(t, src, group=group)
    T = int(t.item())
    buf = torch.empty(2, L, T, hkv, D, dtype=pool_k.dtype, device=pool_k.device)
    dist.recv(buf, src, group=group)
    pages = alloc.alloc((T + ps - 1) // ps)
    if pages is None:
        raise RuntimeError("KV page pool exhausted during receive")
    scatter_pages(pool_k, pool_v, list(pages), buf[0], buf[1])
    return list(pages)
