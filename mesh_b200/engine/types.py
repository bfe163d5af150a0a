"""Serving types with the reference's wire names (serde snake_case).

Restates ``agent/src/inference/engine.rs`` (runtime modes, phases, pause/eviction reasons,
fused kernel stages, decode batch plan) and ``agent/src/inference/job.rs`` (generation config
defaults, request, progress update, segment result, inference result).
"""
from __future__ import annotations

import enum
import time
import uuid
from dataclasses import asdict, dataclass, field
from typing import List, Optional


class _StrEnum(str, enum.Enum):
    def __str__(self):
        return self.value


class InferenceRuntimeMode(_StrEnum):
    FIT_FIRST = "fit_first"
    THROUGHPUT_FIRST = "throughput_first"   # default
    LATENCY_FIRST = "latency_first"
    RESILIENT_EDGE = "resilient_edge"

    @property
    def native(self) -> int:
        return {"fit_first": 0, "throughput_first": 1, "latency_first": 2, "resilient_edge": 3}[self.value]


class ExecutionPhase(_StrEnum):
    PREFILL = "prefill"
    DECODE = "decode"


class KvTransferPolicy(_StrEnum):
    CO_LOCATED = "co_located"
    CHECKPOINT_HANDOFF = "checkpoint_handoff"


class TransportCapabilityTier(_StrEnum):
    RELAY_FALLBACK = "relay_fallback"
    DIRECT_TCP = "direct_tcp"
    DIRECT_PREFERRED = "direct_preferred"
    NVLINK = "nvlink"  # B200 ring members on one NVSwitch fabric


class SessionPauseReason(_StrEnum):
    REGROUP = "regroup"
    FAILOVER = "failover"
    LOCAL_KV_NOT_READY = "local_kv_not_ready"
    RUNTIME_MEMORY_PRESSURE = "runtime_memory_pressure"


class SessionEvictionReason(_StrEnum):
    RUNTIME_MEMORY_PRESSURE = "runtime_memory_pressure"
    IDLE_SESSION = "idle_session"
    COMPLETED_SESSION = "completed_session"


class SessionRuntimeStatus(_StrEnum):
    ACTIVE = "active"
    PAUSED = "paused"
    EVICTED = "evicted"


class BackendOptimizationProfile(_StrEnum):
    CPU_SERIAL = "CpuSerial"
    METAL_VECTORIZED = "MetalVectorized"
    CUDA_FUSED = "CudaFused"
    B200_FUSED = "B200Fused"


class FusedKernelStage(_StrEnum):
    NORM_QKV = "norm_qkv"
    ROPE_KV_WRITE = "rope_kv_write"
    PAGED_ATTENTION = "paged_attention"
    RESIDUAL_MLP = "residual_mlp"
    DEVICE_SAMPLING = "device_sampling"


def _now() -> int:
    return int(time.time())


@dataclass
class DecodeBatchTargets:
    target_session_count: Optional[int] = None
    target_batch_size: Optional[int] = None
    session_ids: List[str] = field(default_factory=list)


@dataclass
class GenerationConfig:
    """Defaults from job.rs:43-54."""
    max_tokens: int = 100
    temperature: float = 0.7
    top_p: float = 0.9
    stop_sequences: List[str] = field(default_factory=list)
    stream: bool = False
    checkpoint_interval: int = 50
    progress_report_interval: int = 4


@dataclass
class InferenceRequest:
    network_id: str
    model_id: str
    prompt_tokens: List[int]
    executor_id: str = ""
    config: GenerationConfig = field(default_factory=GenerationConfig)
    job_id: str = field(default_factory=lambda: str(uuid.uuid4()))
    session_id: str = field(default_factory=lambda: str(uuid.uuid4()))
    phase: ExecutionPhase = ExecutionPhase.PREFILL
    decode_batch_targets: DecodeBatchTargets = field(default_factory=DecodeBatchTargets)
    runtime_mode: InferenceRuntimeMode = InferenceRuntimeMode.THROUGHPUT_FIRST
    fast_path_permitted: bool = True
    created_at: int = field(default_factory=_now)

    def to_dict(self) -> dict:
        d = asdict(self)
        d["phase"] = str(self.phase)
        d["runtime_mode"] = str(self.runtime_mode)
        return d

    @classmethod
    def from_dict(cls, d: dict) -> "InferenceRequest":
        d = dict(d)
        d["config"] = GenerationConfig(**d.get("config", {}))
        d["decode_batch_targets"] = DecodeBatchTargets(**d.get("decode_batch_targets", {}))
        d["phase"] = ExecutionPhase(d.get("phase", "prefill"))
        d["runtime_mode"] = InferenceRuntimeMode(d.get("runtime_mode", "throughput_first"))
        return cls(**d)

    def seed_for_position(self, position: int) -> int:
        """Sampling seed of a token position: job id bits xor position (coordinator.rs:2236)."""
        return (uuid.UUID(self.job_id).int & ((1 << 64) - 1)) ^ position


@dataclass
class InferenceProgressUpdate:
    phase: ExecutionPhase
    completion_tokens: int
    execution_time_ms: int
    time_to_first_token_ms: Optional[int] = None
    kv_cache_seq_len: Optional[int] = None
    batch_size: Optional[int] = None
    active_decode_sessions: Optional[int] = None
    batch_kv_tokens: Optional[int] = None
    deferred_decode_sessions: Optional[int] = None


@dataclass
class InferenceResult:
    job_id: str
    success: bool
    generated_tokens: Optional[List[int]] = None
    error: Optional[str] = None
    prompt_tokens: int = 0
    completion_tokens: int = 0
    execution_time_ms: int = 0
    time_to_first_token_ms: Optional[int] = None
    tokens_per_second: Optional[float] = None
    recovered_from_checkpoint: bool = False

    @classmethod
    def failure(cls, job_id: str, error: str, prompt_tokens: int = 0) -> "InferenceResult":
        return cls(job_id=job_id, success=False, error=error, prompt_tokens=prompt_tokens)


@dataclass
class PrefillComplete:
    job_id: str
    session_id: str
    completion_tokens: int
    execution_time_ms: int
    time_to_first_token_ms: int
    kv_cache_seq_len: int


@dataclass
class DecodeBatchSlot:
    session_id: str
    fairness_epoch: int
    kv_tokens: int


@dataclass
class DecodeBatchPlan:
    slots: List[DecodeBatchSlot]
    deferred: List[str]
    total_kv_tokens: int
    deferred_for_capacity: int = 0
    deferred_for_kv_budget: int = 0
    deferred_for_guardrail: int = 0
