"""Tensor-parallel shard geometry.

The rules match the reference so that shards written by either side are interchangeable:

* attention is split by whole GQA groups (one KV head plus its q heads); groups are dealt out
  as evenly as possible with the remainder going to the lowest positions
  (``scripts/fetch_hf_llama_to_meshnet.py:42-80``; ``agent/src/inference/forward_pass.rs:1257-1315``);
* the MLP intermediate dimension is split into contiguous column ranges of near-equal width,
  remainder to the lowest positions (``artifact_loader.rs:351-366``);
* embedding and final norm are replicated on every rank (``artifact_loader.rs:497-515``).

The column range ``[column_start, column_end)`` recorded in shard metadata is the q-projection
range of the rank, as in the reference (``mesh.column_start`` / ``mesh.column_end``).
"""
from __future__ import annotations

from dataclasses import dataclass

from ..config import ModelConfig


def even_split(total: int, parts: int, index: int) -> tuple[int, int]:
    """Return ``(start, width)`` of part ``index`` when ``total`` items are split into ``parts``
    contiguous ranges whose widths differ by at most one (larger ranges first)."""
    if parts <= 0:
        return 0, total
    base, extra = divmod(total, parts)
    width = base + (1 if index < extra else 0)
    start = index * base + min(index, extra)
    return start, width


@dataclass(frozen=True)
class ShardLayout:
    rank: int
    world: int
    head_dim: int
    q_heads_per_kv_head: int
    kv_head_start: int
    local_kv_heads: int
    q_start: int          # first q column owned (== mesh.column_start)
    q_cols: int
    kv_start: int
    kv_cols: int
    mlp_start: int
    mlp_cols: int

    @property
    def local_q_heads(self) -> int:
        return self.local_kv_heads * self.q_heads_per_kv_head

    @property
    def q_head_start(self) -> int:
        return self.kv_head_start * self.q_heads_per_kv_head

    @property
    def column_start(self) -> int:
        return self.q_start

    @property
    def column_end(self) -> int:
        return self.q_start + self.q_cols


def shard_layout(cfg: ModelConfig, rank: int, world: int) -> ShardLayout:
    cfg.validate()
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"invalid rank {rank} of {world}")
    if world > cfg.num_kv_heads:
        raise ValueError(
            f"TP degree {world} exceeds KV head count {cfg.num_kv_heads}: attention is split by whole GQA groups")
    g0, gn = even_split(cfg.num_kv_heads, world, rank)
    m0, mn = even_split(cfg.intermediate_size, world, rank)
    return ShardLayout(
        rank=rank, world=world, head_dim=cfg.head_dim, q_heads_per_kv_head=cfg.q_heads_per_kv_head,
        kv_head_start=g0, local_kv_heads=gn,
        q_start=g0 * cfg.q_group_width, q_cols=gn * cfg.q_group_width,
        kv_start=g0 * cfg.head_dim, kv_cols=gn * cfg.head_dim,
        mlp_start=m0, mlp_cols=mn,
    )


def validate_column_range(cfg: ModelConfig, column_start: int, column_end: int) -> tuple[int, int]:
    """Validate a q-column range is GQA aligned; return ``(q_cols, kv_cols)``
    (reference ``resolve_attention_shard_widths``, ``artifact_loader.rs:368-408``)."""
    cfg.validate()
    if not 0 <= column_start < column_end <= cfg.hidden_dim:
        raise ValueError(f"Invalid shard range {column_start}..{column_end} for hidden_dim {cfg.hidden_dim}")
    w = cfg.q_group_width
    if column_start % w or column_end % w:
        raise ValueError(f"Shard range {column_start}..{column_end} is not aligned to grouped-query shard width {w}")
    groups = (column_end - column_start) // w
    return column_end - column_start, groups * cfg.head_dim
