"""Pure policy functions restated from the reference control plane.

* consumption quote / settlement: credits = tokens x max(1, model_bytes / GiB / 32)
  (``control-plane/src/consumption_policy.rs:26-65``);
* credit split across assignments: compute share x throughput multiplier (clamped 0.5..1.5,
  relative to the median service rate) x resource-pressure multiplier (0.85 + 0.30 x memory
  pressure), normalised (``credit_policy.rs:49-175``);
* weighted ring column ranges: capacity weight = tier units x memory MB x throughput x stability,
  largest-remainder apportionment, GQA-group granularity with one group reserved per worker
  (``services/ring_manager.rs:131-269``).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Sequence, Tuple

GIB = 1024.0 ** 3
MODEL_SIZE_BUDGET_SCALE_GIB = 32.0
MIN_EXECUTION_TIME_SECS = 0.001
MIN_THROUGHPUT_MULTIPLIER, MAX_THROUGHPUT_MULTIPLIER = 0.5, 1.5
RESOURCE_MULTIPLIER_BASE, RESOURCE_MULTIPLIER_SPAN = 0.85, 0.30
TIER_CAPACITY_UNITS = {"tier0": 1, "tier1": 2, "tier2": 4, "tier3": 8, "tier4": 16}


def model_size_factor(total_model_bytes: int) -> float:
    return max(total_model_bytes / GIB / MODEL_SIZE_BUDGET_SCALE_GIB, 1.0)


def consumption(prompt_tokens: int, completion_tokens: int, total_model_bytes: int) -> dict:
    f = model_size_factor(total_model_bytes)
    p, c = prompt_tokens * f, completion_tokens * f
    return {"model_size_factor": f, "prompt_credits": p, "completion_credits": c, "total_credits": p + c}


def _median(v: List[float]) -> float:
    if not v:
        return 0.0
    v = sorted(v)
    m = len(v) // 2
    return v[m] if len(v) % 2 else (v[m - 1] + v[m]) / 2.0


@dataclass
class AssignmentCreditInput:
    device_id: str
    execution_time_ms: int
    assigned_capacity_units: int
    shard_column_start: int
    shard_column_end: int
    available_memory_bytes: int


def credit_policy(prompt_tokens: int, completion_tokens: int, total_model_bytes: int, total_columns: int,
                  assignments: Sequence[AssignmentCreditInput]) -> dict:
    if not assignments:
        return {"job_credit_budget": 0.0, "assignments": []}
    total_tokens = max(prompt_tokens + completion_tokens, 1)
    budget = total_tokens * model_size_factor(total_model_bytes)
    prep = []
    for a in assignments:
        cols = max(a.shard_column_end - a.shard_column_start, 1)
        frac = cols / max(total_columns, 1)
        units = max(a.assigned_capacity_units, 1) * max(frac, 2.220446049250313e-16)
        secs = max(a.execution_time_ms / 1000.0, MIN_EXECUTION_TIME_SECS)
        rate = units / secs
        est = total_model_bytes * frac
        mp = 1.0 if a.available_memory_bytes == 0 else min(max(est / a.available_memory_bytes, 0.0), 1.0)
        prep.append((a.device_id, units, rate, mp))
    total_units = max(sum(p[1] for p in prep), 2.220446049250313e-16)
    ref_rate = max(_median([p[2] for p in prep]), 2.220446049250313e-16)
    weights = []
    for _, units, rate, mp in prep:
        cs = units / total_units
        tm = min(max(rate / ref_rate, MIN_THROUGHPUT_MULTIPLIER), MAX_THROUGHPUT_MULTIPLIER)
        rm = RESOURCE_MULTIPLIER_BASE + RESOURCE_MULTIPLIER_SPAN * mp
        weights.append((cs, tm, rm, cs * tm * rm))
    total_w = max(sum(w[3] for w in weights), 2.220446049250313e-16)
    out = []
    for (dev, units, rate, mp), (cs, tm, rm, w) in zip(prep, weights):
        share = w / total_w
        out.append({"device_id": dev, "credits": budget * share, "compute_share": cs, "throughput_multiplier": tm,
                    "resource_pressure_multiplier": rm, "normalized_contribution_share": share,
                    "measured_service_rate": rate, "reference_service_rate": ref_rate, "memory_pressure": mp})
    return {"job_credit_budget": budget, "assignments": out}


@dataclass
class CapacityProfile:
    tier: str = "tier2"
    contributed_memory: int = 0
    fallback_memory_mb: int = 1
    throughput_multiplier: float = 1.0
    stability_multiplier: float = 1.0


MIN_RUNTIME_WEIGHT_MULTIPLIER, MAX_RUNTIME_WEIGHT_MULTIPLIER = 0.5, 2.0


def capacity_weight(p: CapacityProfile, tier_units: Dict[str, int] = TIER_CAPACITY_UNITS) -> int:
    mem_mb = max(p.contributed_memory // (1024 * 1024), 1) if p.contributed_memory > 0 else max(p.fallback_memory_mb, 1)
    base = max(tier_units.get(p.tier, 1), 1) * mem_mb
    scaled = base * min(max(p.throughput_multiplier, MIN_RUNTIME_WEIGHT_MULTIPLIER), MAX_RUNTIME_WEIGHT_MULTIPLIER)
    return max(int(round(scaled * min(max(p.stability_multiplier, 0.5), 1.0))), 1)


def weighted_ranges(total: int, weights: Sequence[int]) -> List[Tuple[int, int]]:
    """Largest-remainder apportionment of ``total`` units by weight, contiguous ranges."""
    if not weights:
        return []
    tw = max(sum(weights), 1)
    widths = [(total * w) // tw for w in weights]
    remaining = total - sum(widths)
    rem = sorted(((i, (total * w) % tw) for i, w in enumerate(weights)), key=lambda x: (-x[1], x[0]))
    c = 0
    while remaining > 0:
        widths[rem[c][0]] += 1
        remaining -= 1
        c = (c + 1) % len(rem)
    out, s = [], 0
    for w in widths:
        out.append((s, s + w))
        s += w
    return out


def weighted_group_ranges(total_columns: int, group_width: int, weights: Sequence[int]) -> List[Tuple[int, int]]:
    if group_width <= 0:
        raise ValueError("group_width must be greater than zero")
    if total_columns % group_width:
        raise ValueError(f"tensor parallel dimension {total_columns} is not divisible by grouped-query width {group_width}")
    groups = total_columns // group_width
    if groups >= len(weights):
        bonus = weighted_ranges(groups - len(weights), weights)
        widths = [1 + (e - s) for s, e in bonus]
        r, s = [], 0
        for w in widths:
            r.append((s, s + w))
            s += w
    else:
        r = weighted_ranges(groups, weights)
    return [(a * group_width, b * group_width) for a, b in r]
