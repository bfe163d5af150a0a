"""Model and engine configuration.

``ModelConfig`` mirrors the fields the reference stores in safetensors metadata
(``mesh.hidden_dim`` ... ``mesh.rope_base``; reference ``agent/src/inference/artifact_loader.rs:301-314``
and ``forward_pass.rs:156-190``). ``head_dim`` is ``hidden_dim // num_heads`` exactly as in the
reference (``forward_pass.rs:1280``).

``EngineConfig`` collects the serving knobs: the reference ``InferenceConfig`` defaults
(``coordinator.rs:61-136``) plus the B200 section (TP degree, KV page pool, graph buckets).
"""
from __future__ import annotations

import dataclasses
import os
from dataclasses import dataclass, field
from typing import Optional


@dataclass(frozen=True)
class ModelConfig:
    hidden_dim: int
    num_heads: int
    num_kv_heads: int
    num_layers: int
    vocab_size: int
    intermediate_size: int
    rms_norm_eps: float = 1e-5
    rope_base: float = 10000.0
    name: str = "custom"

    @property
    def head_dim(self) -> int:
        return self.hidden_dim // self.num_heads

    @property
    def q_heads_per_kv_head(self) -> int:
        return self.num_heads // self.num_kv_heads

    @property
    def q_group_width(self) -> int:
        """Columns of the q projection owned by one KV head (one GQA group)."""
        return self.q_heads_per_kv_head * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.num_kv_heads * self.head_dim

    def validate(self) -> None:
        if self.num_heads <= 0 or self.hidden_dim % self.num_heads:
            raise ValueError(f"hidden_dim {self.hidden_dim} not divisible by num_heads {self.num_heads}")
        if self.num_kv_heads <= 0 or self.num_heads % self.num_kv_heads:
            raise ValueError(f"num_heads {self.num_heads} not divisible by num_kv_heads {self.num_kv_heads}")
        if self.head_dim % 2:
            raise ValueError("RoPE requires an even head_dim")

    def param_count(self) -> int:
        h, i, v = self.hidden_dim, self.intermediate_size, self.vocab_size
        per_layer = h * h * 2 + 2 * h * self.kv_dim + 3 * h * i + 2 * h
        return self.num_layers * per_layer + 2 * v * h + h

    def to_metadata(self, model_id: str) -> dict:
        return {
            "mesh.model_id": model_id,
            "mesh.hidden_dim": str(self.hidden_dim),
            "mesh.num_heads": str(self.num_heads),
            "mesh.num_kv_heads": str(self.num_kv_heads),
            "mesh.num_layers": str(self.num_layers),
            "mesh.vocab_size": str(self.vocab_size),
            "mesh.intermediate_size": str(self.intermediate_size),
            "mesh.rms_norm_eps": str(self.rms_norm_eps),
            "mesh.rope_base": str(self.rope_base),
        }

    @classmethod
    def from_metadata(cls, md: dict) -> "ModelConfig":
        def req(k):
            if k not in md:
                raise KeyError(f"Missing safetensors metadata key {k}")
            return md[k]
        return cls(
            hidden_dim=int(req("mesh.hidden_dim")),
            num_heads=int(req("mesh.num_heads")),
            num_kv_heads=int(req("mesh.num_kv_heads")),
            num_layers=int(req("mesh.num_layers")),
            vocab_size=int(req("mesh.vocab_size")),
            intermediate_size=int(req("mesh.intermediate_size")),
            rms_norm_eps=float(req("mesh.rms_norm_eps")),
            rope_base=float(req("mesh.rope_base")),
            name=md.get("mesh.model_id", "custom"),
        )

    def replace(self, **kw) -> "ModelConfig":
        return dataclasses.replace(self, **kw)


PRESETS = {
    # TinyLlama-1.1B shape (the CPU TP=2 loopback configuration)
    "tinyllama-1.1b": ModelConfig(2048, 32, 4, 22, 32000, 5632, 1e-5, 1e4, "tinyllama-1.1b"),
    # Llama-3-8B shape (headline serving configuration and the prefill sweep)
    "llama3-8b": ModelConfig(4096, 32, 8, 32, 128256, 14336, 1e-5, 5e5, "llama3-8b"),
    # Llama-3-70B shape (TP=8 serving with mid-run KV handoff)
    "llama3-70b": ModelConfig(8192, 64, 8, 80, 128256, 28672, 1e-5, 5e5, "llama3-70b"),
    # reference default ModelConfig (forward_pass.rs:174-186)
    "reference-default": ModelConfig(8192, 64, 8, 80, 32000, 28672, 1e-5, 1e4, "reference-default"),
    # small shapes for tests: head_dim 64/128, GQA 4, MLP multiple of 64 per rank at TP<=4
    "tiny": ModelConfig(512, 4, 2, 2, 512, 512, 1e-5, 1e4, "tiny"),
    "tiny-gqa": ModelConfig(1024, 8, 2, 2, 1024, 1024, 1e-5, 5e5, "tiny-gqa"),
    "small": ModelConfig(1024, 8, 2, 4, 4096, 2816, 1e-5, 5e5, "small"),
}


def get_preset(name: str) -> ModelConfig:
    try:
        return PRESETS[name]
    except KeyError as exc:
        raise KeyError(f"unknown model preset {name!r}; known: {sorted(PRESETS)}") from exc


@dataclass
class EngineConfig:
    """Serving configuration (reference ``InferenceConfig``, ``coordinator.rs:61-136``)."""

    # reference defaults
    allreduce_timeout_s: float = 30.0
    job_timeout_s: float = 300.0
    checkpoint_segment_max_tokens: int = 1024
    max_decode_batch_size: int = 4
    max_decode_batch_kv_tokens: int = 16384
    max_active_sessions: int = 8
    kv_memory_budget_bytes: int = 512 * 1024 * 1024
    runtime_memory_budget_bytes: int = 2 * 1024 * 1024 * 1024
    recovery_cooldown_s: float = 5.0
    recovery_max_loads_per_minute: int = 8
    runtime_mode: str = "throughput_first"
    # KV paging (reference DEFAULT_LIVE_KV_PAGE_TOKENS = 16, kv_cache.rs:191-221)
    page_size: int = 16
    num_pages: int = 0  # 0 = size from max_sessions * max_seq_len
    max_seq_len: int = 8192
    # compat: reference keeps a 4096-token sliding window (forward_pass.rs:1795); None = exact
    sliding_window: Optional[int] = None
    # B200 section
    tp: int = 1
    dtype: str = "bf16"
    use_cuda_graphs: bool = True
    decode_batch_buckets: tuple = (1, 2, 4, 8, 16, 32, 64, 128, 256)
    prefill_chunk_tokens: int = 16384
    use_fused_allreduce: bool = True
    # auto: the separate peer-memory all-reduce + residual + RMSNorm kernel after the o_proj / down
    # GEMM, one-shot or two-shot by size (unfused: the same); gemm_ar: decode steps run the
    # all-reduce inside the GEMM's launch; oneshot | twoshot | push | push_oneshot | nccl: that
    # all-reduce everywhere
    allreduce_impl: str = "auto"
    # allow the fused all-reduce to use NVSwitch NVLS (multimem loads/stores) when the node has it;
    # it is used from 8 ranks up, where it measured faster (TP8 decode 23.98k vs 22.74k tok/s),
    # while 2 ranks measured equal and plain peer loads stay the default below 8
    nvls: bool = True
    # TP prefill: run a chunk of several prompts as two halves on two streams so one half's
    # all-reduces overlap the other half's GEMMs (each half needs >= 512 tokens)
    prefill_overlap: bool = field(default_factory=lambda: os.environ.get("MESH_PREFILL_OVERLAP", "0") == "1")
    extra: dict = field(default_factory=dict)

    def bucket_for(self, batch: int) -> int:
        for b in self.decode_batch_buckets:
            if batch <= b:
                return b
        raise ValueError(f"decode batch {batch} exceeds largest bucket {self.decode_batch_buckets[-1]}")
