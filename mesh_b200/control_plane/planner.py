"""Execution planner: which ring members serve the prefill and the decode phase of a request.

Restates ``control-plane/src/services/planner.rs``:

* only workers whose backend contract supports production serving are planned (``:669-675``);
* the runtime mode comes from the members: any relayed or degraded link -> ``resilient_edge``;
  a capacity spread of 4x or more -> ``throughput_first``; else ``latency_first`` (``:1215-1247``);
* for each phase, candidate groups are built per execution island (workers sharing a fast-path
  contract hash) and per layout rule (the canonical tensor-parallel tiling, full-replica sets of
  every allowed size ordered by the mode, contiguous pipeline windows, hybrid windows whose stage
  chunks tile the columns), filtered by the layout rules, and the best-scoring one wins
  (``:689-1001``);
* the score is effective capacity x 100 + a transport bonus + capacity balance - a collective
  scale risk - a width penalty per mode; decode additionally penalises groups wider than a
  narrower candidate that covers the same shape unless they beat it by a margin (180, or 320 for
  models of at most 16 GiB), and mixed-provider groups when a homogeneous one is nearly as good
  (``:1258-1560``);
* the KV owner is the member with the most capacity units, then memory, then the lowest ring
  position (``:677-688``);
* decode groups differing from the prefill group use ``checkpoint_handoff`` KV transfer, else
  ``co_located``;
* re-planning a decode group keeps the current one unless the new choice is better by the margin
  (hysteresis), and never widens a full-replica group (``:203-372``).
"""
from __future__ import annotations

import uuid
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence

from .layout import LayoutError, LayoutRule, Member, ModelManifest, validate_group

RUNTIME_MODES = ("fit_first", "throughput_first", "latency_first", "resilient_edge")
MIN_RUNTIME_CAPACITY_MULTIPLIER = 0.5
MAX_RUNTIME_CAPACITY_MULTIPLIER = 2.0
SMALL_MODEL_EXPANSION_THRESHOLD_BYTES = 16 * 1024 ** 3
EXPANSION_SCORE_MARGIN = 180
SMALL_MODEL_EXPANSION_SCORE_MARGIN = 320


class PlanningError(RuntimeError):
    """No legal group can be formed (HTTP 409)."""


# ---------------------------------------------------------------------------------------------- basics
def production_members(members: Sequence[Member]) -> List[Member]:
    return [m for m in members if m.backend_contract.supports_production_serving()]


def _degraded(m: Member) -> bool:
    if m.connectivity_status is None:
        return True
    return m.connectivity_status != "connected" or m.active_path == "relay"


def derive_runtime_mode(members: Sequence[Member]) -> str:
    if any(_degraded(m) for m in members):
        return "resilient_edge"
    caps = [max(1, m.assigned_capacity_units) for m in members] or [1]
    lo, hi = min(caps), max(caps)
    return "throughput_first" if hi >= max(lo * 4, 4) else "latency_first"


def adjusted_capacity_units(base_units: int, throughput_multiplier: float) -> int:
    f = min(max(throughput_multiplier, MIN_RUNTIME_CAPACITY_MULTIPLIER), MAX_RUNTIME_CAPACITY_MULTIPLIER)
    return max(1, int(round(max(1, base_units) * f)))


def transport_tier(members: Sequence[Member]) -> str:
    dataplane = all(any(a.startswith("dataplane://") for a in m.listen_addrs) for m in members)
    if dataplane and all(m.connectivity_status == "connected" and m.active_path == "direct" for m in members):
        return "direct_preferred"
    return "direct_tcp" if dataplane else "relay_fallback"


def select_kv_owner(members: Sequence[Member]) -> str:
    best = max(members, key=lambda m: (m.assigned_capacity_units, m.contributed_memory, -m.ring_position))
    return best.device_id


def same_participants(a: Sequence[Member], b: Sequence[Member]) -> bool:
    return sorted(m.device_id for m in a) == sorted(m.device_id for m in b)


def is_full_replica_group(members: Sequence[Member]) -> bool:
    if not members:
        return False
    top = max(m.column_end for m in members)
    return all(m.column_start == 0 and m.column_end == top for m in members)


def is_homogeneous(members: Sequence[Member]) -> bool:
    return len({m.backend_contract.contract_hash for m in members}) <= 1


# ---------------------------------------------------------------------------------------------- scoring
def _throughput_spread_penalty(members: Sequence[Member]) -> int:
    xs = sorted(m.throughput_multiplier for m in members
                if m.throughput_multiplier is not None and m.throughput_multiplier > 0)
    if len(xs) < 2 or xs[-1] <= 1e-12:
        return 0
    return max(0, int(round((1.0 - min(max(xs[0] / xs[-1], 0.0), 1.0)) * 90.0)))


def _avg_ratio_penalty(vals: Sequence[float], scale: float) -> int:
    if not vals:
        return 0
    avg = sum(vals) / len(vals)
    return max(0, int(round(min(max(avg, 0.0), 1.0) * scale)))


def _avg_fill_penalty(vals: Sequence[float]) -> int:
    if not vals:
        return 0
    avg = sum(vals) / len(vals)
    return max(0, int(round((1.0 - min(max(avg, 0.0), 1.0)) * 140.0)))


def collective_scale_risk(members: Sequence[Member], tier: str) -> int:
    if not members:
        return 100
    width = len(members)
    caps = [max(1, m.assigned_capacity_units) for m in members]
    lo, hi = min(caps), max(caps)
    degraded = sum(1 for m in members if _degraded(m))
    provider_mix = (len({m.backend_contract.contract_hash for m in members}) - 1) * 15
    transport = {"direct_preferred": 0, "direct_tcp": 15, "relay_fallback": 40}[tier]
    width_pen = max(0, width - 2) * 12
    balance = 100 - max(1, lo * 100 // hi)
    instability = sum(m.instability_score for m in members)
    deferral = _avg_ratio_penalty([m.observed_deferred_ratio for m in members
                                   if m.observed_deferred_ratio is not None], 120.0)
    fill = _avg_fill_penalty([m.observed_fill_ratio for m in members
                              if m.observed_fill_ratio is not None]) if width > 2 else 0
    return (width_pen + balance + degraded * 25 + provider_mix + transport + instability +
            _throughput_spread_penalty(members) + deferral + fill)


def topology_efficiency_score(members: Sequence[Member], mode: str) -> int:
    if not members:
        return -(1 << 61)
    width = len(members)
    caps = [max(1, m.assigned_capacity_units) for m in members]
    total, lo, hi = sum(caps), min(caps), max(caps)
    aligned = lo * width
    excess = max(0, total - aligned)
    tier = transport_tier(members)
    risk = collective_scale_risk(members, tier)
    divisor = 2 if width <= 2 else 4 + risk // 25
    effective = aligned + excess // max(1, divisor)
    bonus = {"direct_preferred": 160, "direct_tcp": 80, "relay_fallback": 0}[tier]
    balance = min(max(lo * 100 // max(1, hi), 1), 100)
    if mode == "throughput_first":
        wpen = 0 if width <= 2 else (width - 2) * 35
    else:
        wpen = max(0, width - 1) * {"latency_first": 70, "fit_first": 45, "resilient_edge": 20}[mode]
    return effective * 100 + bonus + balance - risk - wpen


def _covers_same_decode_shape(cand: Sequence[Member], ref: Sequence[Member], everyone: Sequence[Member]) -> bool:
    if is_full_replica_group(cand) and is_full_replica_group(ref):
        return True
    full = max((m.column_end for m in everyone), default=0)
    span = lambda g: sum(max(0, m.column_end - m.column_start) for m in g)  # noqa: E731
    return span(cand) >= full and span(ref) >= full


def scored_candidate(manifest: ModelManifest, phase: str, mode: str, everyone: Sequence[Member],
                     valid: Sequence[Sequence[Member]], cand: Sequence[Member]) -> int:
    score = topology_efficiency_score(cand, mode)
    if phase != "decode":
        return score
    width = len(cand)
    narrower = [o for o in valid if len(o) < width]
    best_narrow = max((topology_efficiency_score(o, mode) for o in narrower), default=None)
    best_homog = max((topology_efficiency_score(o, mode) for o in valid if is_homogeneous(o)), default=None)
    small = manifest.total_model_bytes <= SMALL_MODEL_EXPANSION_THRESHOLD_BYTES
    wider_than_needed = any(_covers_same_decode_shape(o, cand, everyone) for o in narrower)
    if small and width > 2 and wider_than_needed:
        score -= (width - 2) * 180
    if best_narrow is not None:
        margin = SMALL_MODEL_EXPANSION_SCORE_MARGIN if small else EXPANSION_SCORE_MARGIN
        if width > 1 and wider_than_needed and score < best_narrow + margin:
            score -= 5000
    if not is_homogeneous(cand) and wider_than_needed and best_homog is not None and best_homog + 120 >= score:
        score -= 2000
    return score


# ---------------------------------------------------------------------------------------------- candidates
def _rank(members: Sequence[Member]) -> List[Member]:
    return sorted(members, key=lambda m: (-m.assigned_capacity_units, -m.contributed_memory, m.ring_position))


def _full_replicas(members: Sequence[Member], dim: int) -> List[Member]:
    return [m for m in members if m.column_start == 0 and m.column_end == dim]


def canonical_tensor_parallel_group(members: Sequence[Member], dim: int) -> Optional[List[Member]]:
    """Walk the columns from 0: at each cursor take the member starting there (most capacity, then
    memory, on ties); None if the walk cannot reach ``dim``."""
    ranked = sorted(members, key=lambda m: (m.column_start, m.column_end, -m.assigned_capacity_units,
                                            -m.contributed_memory))
    cursor, out = 0, []
    while cursor < dim:
        nxt = next((m for m in ranked if m.column_start == cursor and m.column_end > cursor), None)
        if nxt is None:
            return None
        out.append(nxt)
        cursor = nxt.column_end
    return out


def _ordered_sizes(available: int, lo: Optional[int], hi: Optional[int], mode: str) -> List[int]:
    lo = lo or 1
    upper = min(hi if hi is not None else available, available)
    if lo > upper:
        return []
    sizes = list(range(lo, upper + 1))
    return sorted(sizes, reverse=(mode == "throughput_first"))


def _windows(members: Sequence[Member], width: int) -> List[List[Member]]:
    if width <= 0 or len(members) < width:
        return []
    return [list(members[i:i + width]) for i in range(len(members) - width + 1)]


def _tiles_columns(members: Sequence[Member], dim: int) -> bool:
    cursor = 0
    for m in sorted(members, key=lambda m: (m.column_start, m.column_end)):
        if m.column_start != cursor or m.column_end <= m.column_start:
            return False
        cursor = m.column_end
    return cursor == dim


def candidates_for_rule(manifest: ModelManifest, members: Sequence[Member], mode: str,
                        rule: LayoutRule) -> List[List[Member]]:
    dim = manifest.tensor_parallelism_dim
    if rule.layout == "tensor_parallel":
        g = canonical_tensor_parallel_group(members, dim)
        if g and (rule.tensor_parallel_degree is None or rule.tensor_parallel_degree == len(g)):
            return [g]
        return []
    if rule.layout == "full_replica":
        reps = _rank(_full_replicas(members, dim))
        return [reps[:n] for n in _ordered_sizes(len(reps), rule.min_members, rule.max_members, mode)
                if 0 < n <= len(reps)]
    if rule.layout == "pipeline":
        if rule.pipeline_parallel_degree is None:
            return []
        reps = sorted(_full_replicas(members, dim), key=lambda m: m.ring_position)
        return _windows(reps, rule.pipeline_parallel_degree)
    pp, tp = rule.pipeline_parallel_degree, rule.tensor_parallel_degree
    if not pp or not tp:
        return []
    ordered = sorted(members, key=lambda m: m.ring_position)
    return [w for w in _windows(ordered, pp * tp)
            if all(_tiles_columns(w[s * tp:(s + 1) * tp], dim) for s in range(pp))]


def execution_islands(members: Sequence[Member]) -> Dict[tuple, List[Member]]:
    """Fast-path-eligible members grouped by (compatibility class, contract hash)."""
    out: Dict[tuple, List[Member]] = {}
    for m in members:
        c = m.backend_contract
        if c.fast_path_eligible:
            out.setdefault((c.compatibility_class, c.contract_hash), []).append(m)
    return dict(sorted(out.items()))


def island_id(model_id: str, phase: str, members: Sequence[Member]) -> str:
    hashes = {m.backend_contract.contract_hash for m in members}
    if len(hashes) != 1 or not all(m.backend_contract.fast_path_eligible for m in members):
        raise PlanningError(f"production execution island for model {model_id} phase {phase} must be "
                            f"homogeneous fast-path")
    c = members[0].backend_contract
    return f"island:{model_id}:{phase}:{c.compatibility_class}:{c.contract_hash}".lower()


def candidate_groups(manifest: ModelManifest, phase: str, members: Sequence[Member], mode: str) -> List[List[Member]]:
    out: List[List[Member]] = []
    seen = set()
    for island in execution_islands(members).values():
        for rule in manifest.rules_for(phase):
            for cand in candidates_for_rule(manifest, island, mode, rule):
                cand = sorted(cand, key=lambda m: m.ring_position)
                key = tuple(m.device_id for m in cand)
                if cand and key not in seen:
                    seen.add(key)
                    out.append(cand)
    if phase == "decode" and mode == "throughput_first":
        order = {"direct_preferred": 2, "direct_tcp": 1, "relay_fallback": 0}
        out.sort(key=lambda g: (topology_efficiency_score(g, mode), order[transport_tier(g)],
                                sum(max(1, m.assigned_capacity_units) for m in g), -len(g)), reverse=True)
    return out


def select_execution_members(manifest: ModelManifest, phase: str, members: Sequence[Member],
                             mode: str) -> List[Member]:
    if not members:
        raise PlanningError(f"no production-serving members are available for model {manifest.model_id} "
                            f"phase {phase}")
    valid, errors = [], []
    for cand in candidate_groups(manifest, phase, members, mode):
        try:
            validate_group(manifest, phase, cand)
            valid.append(cand)
        except LayoutError as e:
            errors.append(str(e))
    if not valid:
        raise PlanningError(f"no execution-valid {phase} group could be formed for model {manifest.model_id}: "
                            + "; ".join(errors))
    # max by score; the first of equal scores wins (candidate order is deterministic)
    best, best_s = None, None
    for cand in valid:
        s = scored_candidate(manifest, phase, mode, members, valid, cand)
        if best_s is None or s > best_s:
            best, best_s = cand, s
    return best


# ---------------------------------------------------------------------------------------------- plans
@dataclass
class Plan:
    plan_id: str
    runtime_mode: str
    prefill: List[Member]
    decode: List[Member]
    prefill_island: str
    decode_island: str

    @property
    def kv_transfer_policy(self) -> str:
        return "co_located" if same_participants(self.prefill, self.decode) else "checkpoint_handoff"

    def to_json(self, model_id: str, session_id: str) -> dict:
        groups = []
        for phase, members, isl in (("prefill", self.prefill, self.prefill_island),
                                    ("decode", self.decode, self.decode_island)):
            groups.append({
                "group_id": f"group-{self.plan_id}-{phase}", "phase": phase, "model_id": model_id,
                "execution_island_id": isl, "transport_tier": transport_tier(members),
                "kv_transfer_policy": "co_located" if phase == "prefill" else self.kv_transfer_policy,
                "total_capacity_units": sum(m.assigned_capacity_units for m in members),
                "backend_contract_hash": members[0].backend_contract.contract_hash,
                "members": [dict(m.to_json(), total_workers=len(members)) for m in members]})
        segs = [{"segment_id": f"segment-{session_id}-{g['phase']}", "phase": g["phase"],
                 "execution_group_id": g["group_id"], "session_id": session_id,
                 "kv_owner_device_id": select_kv_owner(mm),
                 "participant_device_ids": [m.device_id for m in mm]}
                for g, mm in zip(groups, (self.prefill, self.decode))]
        return {"plan_id": self.plan_id, "model_id": model_id, "runtime_mode": self.runtime_mode,
                "execution_groups": groups, "segments": segs, "initial_segment_id": segs[0]["segment_id"],
                "kv_owner_device_id": segs[0]["kv_owner_device_id"],
                "kv_transfer_policy": self.kv_transfer_policy}


def plan(manifest: ModelManifest, members: Sequence[Member], runtime_mode: Optional[str] = None) -> Plan:
    prod = production_members(members)
    if not prod:
        raise PlanningError(f"no production-serving workers are available for model {manifest.model_id}")
    mode = runtime_mode or derive_runtime_mode(prod)
    pre = select_execution_members(manifest, "prefill", prod, mode)
    dec = select_execution_members(manifest, "decode", prod, mode)
    return Plan(str(uuid.uuid4()), mode, pre, dec, island_id(manifest.model_id, "prefill", pre),
                island_id(manifest.model_id, "decode", dec))


def refresh_decode_plan(manifest: ModelManifest, current: Plan, members: Sequence[Member]) -> Plan:
    """Re-select the decode group on the live topology; keep the current group unless the new one
    is materially better (hysteresis), and never replace a full-replica group by a wider one."""
    prod = production_members(members)
    if not prod:
        raise PlanningError(f"live topology no longer has any production-serving workers for model "
                            f"{manifest.model_id}")
    mode = derive_runtime_mode(prod)
    chosen = select_execution_members(manifest, "decode", prod, mode)
    present = {m.device_id: m for m in prod}
    cur = None
    if all(m.device_id in present for m in current.decode):
        cur = [present[m.device_id] for m in current.decode]
        try:
            validate_group(manifest, "decode", cur)
        except LayoutError:
            cur = None
    if cur is not None:
        if len(chosen) > len(cur) and is_full_replica_group(cur):
            chosen = cur
        else:
            both = [chosen, cur]
            s_new = scored_candidate(manifest, "decode", mode, members, both, chosen)
            s_cur = scored_candidate(manifest, "decode", mode, members, both, cur)
            margin = (SMALL_MODEL_EXPANSION_SCORE_MARGIN if manifest.total_model_bytes <=
                      SMALL_MODEL_EXPANSION_THRESHOLD_BYTES else EXPANSION_SCORE_MARGIN)
            if same_participants(chosen, cur) or s_new < s_cur + margin:
                chosen = cur
    return Plan(current.plan_id, mode, current.prefill, chosen, current.prefill_island,
                island_id(manifest.model_id, "decode", chosen))
