"""Inference statistics with the reference's JSON keys (``agent/src/inference/stats.rs:19-249``),
persisted to ``$MESHNET_HOME/inference_stats.json`` (``stats.rs:2233-2237``), plus B200-specific
device-timed fields (per-phase milliseconds measured with CUDA events)."""
from __future__ import annotations

import json
import os
import threading
import time
from pathlib import Path
from typing import Dict

COUNTERS = (
    "jobs_completed jobs_failed total_tokens_generated total_prompt_tokens total_inference_time_ms "
    "total_allreduce_time_ms decode_microbatches_executed decode_sessions_batched "
    "decode_multi_session_microbatches decode_batch_size_peak decode_batch_kv_tokens_total "
    "decode_batch_deferred_sessions decode_batch_capacity_deferrals decode_batch_kv_budget_deferrals "
    "decode_batch_guardrail_deferrals prefill_fast_path_plans decode_fast_path_plans fast_path_arena_reuses "
    "fast_path_layout_validated_plans fast_path_replay_preferred_plans fast_path_decode_bucket_batch_ceiling_peak "
    "fast_path_decode_bucket_token_ceiling_peak fast_path_prefill_token_ceiling_peak checkpoints_created "
    "checkpoint_recoveries recovery_attempts recovery_cooldown_rejections recovery_budget_rejections "
    "recovery_checkpoint_misses allreduce_operations total_layers_processed tensor_bytes_sent tensor_bytes_received "
    "tensor_reduce_scatter_bytes_sent tensor_reduce_scatter_bytes_received tensor_all_gather_bytes_sent "
    "tensor_all_gather_bytes_received tensor_barrier_bytes_sent tensor_barrier_bytes_received "
    "tensor_bulk_transfer_bytes_sent tensor_bulk_transfer_bytes_received tensor_checkpoint_bytes_sent "
    "tensor_checkpoint_bytes_received tensor_send_count tensor_send_latency_ms tensor_receive_count "
    "tensor_receive_latency_ms tensor_send_timeout_count tensor_receive_timeout_count "
    "total_reduce_scatter_time_ms total_all_gather_time_ms total_collective_operations "
    "total_collective_worker_participants total_collective_bytes_sent total_collective_bytes_received "
    "total_device_resident_collectives kv_snapshot_exports kv_snapshot_export_bytes kv_snapshot_materializations "
    "kv_snapshot_materialized_bytes device_sampling_requests device_sampling_fallback_requests "
    "host_sampling_requests total_sampling_time_ms device_sampling_time_ms host_sampling_time_ms "
    # B200 additions
    "cuda_graph_replays cuda_graph_captures device_prefill_time_ms device_decode_time_ms "
    "fused_allreduce_operations nccl_allreduce_operations kernel_launches"
).split()
PEAKS = {"decode_batch_size_peak", "fast_path_decode_bucket_batch_ceiling_peak",
         "fast_path_decode_bucket_token_ceiling_peak", "fast_path_prefill_token_ceiling_peak"}


class InferenceStats:
    def __init__(self):
        self._lock = threading.Lock()
        self.values: Dict[str, float] = {k: 0 for k in COUNTERS}
        self.values["start_time"] = int(time.time())

    def add(self, key: str, v: float = 1) -> None:
        with self._lock:
            if key in PEAKS:
                self.values[key] = max(self.values.get(key, 0), v)
            else:
                self.values[key] = self.values.get(key, 0) + v

    def get(self, key: str) -> float:
        return self.values.get(key, 0)

    def derived(self) -> dict:
        v = self.values
        up = max(1e-9, time.time() - v["start_time"])
        t = v["total_inference_time_ms"]
        return {
            "avg_tokens_per_second": (v["total_tokens_generated"] / (t / 1e3)) if t else 0.0,
            "uptime_seconds": up,
            "avg_decode_batch_size": (v["decode_sessions_batched"] / v["decode_microbatches_executed"])
            if v["decode_microbatches_executed"] else 0.0,
            "avg_allreduce_time_ms": (v["total_allreduce_time_ms"] / v["allreduce_operations"])
            if v["allreduce_operations"] else 0.0,
        }

    def snapshot(self) -> dict:
        with self._lock:
            d = dict(self.values)
        d.update(self.derived())
        return d

    def save_to_file(self, home: str = "") -> Path:
        base = Path(home or os.environ.get("MESHNET_HOME", str(Path.home() / ".meshnet")))
        base.mkdir(parents=True, exist_ok=True)
        p = base / "inference_stats.json"
        tmp = p.with_suffix(".json.tmp")
        tmp.write_text(json.dumps(self.snapshot(), indent=2, sort_keys=True))
        tmp.replace(p)
        return p

    @classmethod
    def load(cls, path: Path) -> "InferenceStats":
        s = cls()
        s.values.update(json.loads(Path(path).read_text()))
        return s
