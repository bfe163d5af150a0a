"""Claim-time scheduler: which assignment a worker gets when it asks for work.

Restates ``control-plane/src/services/scheduler.rs``:

* four policy modes, ``fit_first``, ``throughput_first``, ``latency_first``, ``resilient_edge``
  (``:19-25``);
* order of a claim: an in-flight prefill group the worker belongs to; then a prefill whose decode
  cohort is already waiting; then the best runnable candidate by rank (``:119-197``);
* every candidate is first classified: runnable (with its ready time) or blocked with a reason,
  ``queue_missing``, ``waiting_for_transfer``, ``waiting_for_prefill_cohort``,
  ``lease_held_by_peer``, ``already_running`` or ``not_eligible`` (``:362-550``);
* the rank is a lexicographic key: coordination (prefill groups already in flight first, then new
  prefill, then decode), fairness soft caps (submitter active jobs, model active jobs against
  workers / divisor, model active capacity against capacity units / divisor), the runtime mode's
  priority, the policy mode's own key (decode cohort fill, cohort age, leased-assignment counts,
  created / ready time), the session order and, for throughput-first decode, the topology rank
  (``:552-935``).
Times are ISO-8601 strings (compared lexicographically, as in the reference).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple, Union

MODES = ("fit_first", "throughput_first", "latency_first", "resilient_edge")
BLOCKED_REASONS = ("queue_missing", "waiting_for_transfer", "waiting_for_prefill_cohort", "lease_held_by_peer",
                   "already_running", "not_eligible")
FAR_FUTURE = "9999-12-31T23:59:59Z"


@dataclass
class Candidate:
    """One assignment the requesting worker could take (the scheduler's view of the DB rows)."""
    assignment_id: str
    job_id: str
    session_id: str
    phase: str                                   # prefill | decode
    group_status: str                            # prefill_member, prefill_leased, prefill_active, decode_*
    model_id: str = "m"
    ring_position: int = 0
    runtime_mode: str = "throughput_first"
    submitted_by_device_id: str = ""
    created_at: str = ""
    assigned_at: str = ""
    decode_queue_status: Optional[str] = None    # blocked_on_prefill, blocked_on_transfer, ready, leased, ...
    decode_ready_at: Optional[str] = None
    decode_lease_owner_device_id: Optional[str] = None
    decode_lease_expires_at: Optional[str] = None
    decode_updated_at: Optional[str] = None
    group_lease_owner_device_id: Optional[str] = None
    group_lease_expires_at: Optional[str] = None
    prefill_group_total_members: int = 1
    prefill_group_leased_members: int = 0
    prefill_group_active_members: int = 0
    model_prefill_inflight_groups: int = 0
    foreign_transport_island_inflight_jobs: int = 0
    decode_lease_target_session_count: Optional[int] = None
    decode_cohort_ready_sessions: int = 0
    decode_cohort_blocked_sessions: int = 0
    decode_cohort_blocked_prefill_sessions: int = 0
    decode_cohort_oldest_ready_at: Optional[str] = None
    decode_cohort_leased_sessions: int = 0
    decode_cohort_active_sessions: int = 0
    decode_topology_rank: int = 0


@dataclass
class Blocked:
    session_id: str
    job_id: str
    assignment_id: str
    reason: str


@dataclass
class Runnable:
    candidate: Candidate
    ready_at: str


@dataclass
class SchedulingPolicy:
    submitter_active_job_soft_cap: int = 1
    model_active_job_soft_cap_divisor: int = 2
    capacity_unit_soft_cap_divisor: int = 2


@dataclass
class Snapshot:
    active_jobs_by_submitter: Dict[str, int] = field(default_factory=dict)
    active_jobs_by_model: Dict[str, int] = field(default_factory=dict)
    active_capacity_by_model: Dict[str, int] = field(default_factory=dict)
    leased_assignments_by_submitter: Dict[str, int] = field(default_factory=dict)
    leased_assignments_by_job: Dict[str, int] = field(default_factory=dict)
    online_worker_count: int = 1
    online_capacity_units: int = 1


@dataclass
class Decision:
    selected_assignment_id: Optional[str]
    blocked: List[Blocked]


# ---------------------------------------------------------------------------------------------- classify
def should_wait_for_prefill_cohort(c: Candidate) -> bool:
    if c.phase != "decode" or c.decode_cohort_blocked_prefill_sessions == 0:
        return False
    fill = c.decode_cohort_ready_sessions + c.decode_cohort_leased_sessions + c.decode_cohort_active_sessions
    total = fill + c.decode_cohort_blocked_sessions
    target = max(c.decode_lease_target_session_count or 0, total, 1)
    return fill < target and c.decode_cohort_leased_sessions == 0 and c.decode_cohort_active_sessions == 0


_ATTACHABLE = ("decode_ready", "decode_member", "decode_leased")


def classify(c: Candidate, requesting_device_id: str, now: str) -> Union[str, Tuple[str]]:
    """Ready time (str) of a runnable candidate, or a 1-tuple holding the blocked reason."""
    if c.phase == "prefill":
        if c.group_status in ("prefill_member", "prefill_leased"):
            inflight = c.prefill_group_leased_members + c.prefill_group_active_members
            if inflight > 0:
                return c.created_at
            if c.foreign_transport_island_inflight_jobs > 0 or c.model_prefill_inflight_groups > 0 \
                    or c.ring_position != 0:
                return ("lease_held_by_peer",)
            return c.created_at
        if c.group_status == "prefill_active":
            return ("already_running",)
        return ("not_eligible",)
    q = c.decode_queue_status
    if q is None:
        return ("queue_missing",)
    attachable_peer = q in ("leased", "active") and c.group_status in _ATTACHABLE + ("decode_active",)
    if c.foreign_transport_island_inflight_jobs > 0 and not attachable_peer:
        return ("lease_held_by_peer",)
    member_states = ("decode_member", "decode_leased", "decode_active")
    peer_active_cohort = c.decode_cohort_active_sessions > 0 and c.group_status not in member_states
    peer_prefill_inflight = c.model_prefill_inflight_groups > 0 and c.group_status not in member_states
    wait_prefill = should_wait_for_prefill_cohort(c)
    ready_time = c.decode_ready_at or c.decode_updated_at or c.created_at
    if q == "blocked_on_transfer":
        return ("waiting_for_transfer",)
    if q == "active":
        if c.group_status == "decode_pending_transfer":
            return ("waiting_for_transfer",)
        owner = c.group_lease_owner_device_id or c.decode_lease_owner_device_id
        if owner is not None and owner != requesting_device_id and c.group_status in _ATTACHABLE:
            return ready_time
        return ("already_running",)
    if q in ("completed", "failed"):
        return ("not_eligible",)
    if q in ("leased", "ready"):
        if peer_prefill_inflight or peer_active_cohort:
            return ("lease_held_by_peer",)
        if q == "leased":
            owner = c.group_lease_owner_device_id or c.decode_lease_owner_device_id
            expires = c.group_lease_expires_at or c.decode_lease_expires_at
        else:
            owner, expires = c.group_lease_owner_device_id, c.group_lease_expires_at
        held = owner is not None and owner != requesting_device_id and expires is not None and expires > now
        if held and c.group_status not in _ATTACHABLE:
            return ("lease_held_by_peer",)
        if c.group_status == "decode_pending_transfer":
            return ("waiting_for_transfer",)
        if wait_prefill:
            return ("waiting_for_prefill_cohort",)
        if c.group_status in _ATTACHABLE:
            return ready_time
        return ("not_eligible",)
    return ("not_eligible",)


# ---------------------------------------------------------------------------------------------- rank
def coordination_rank(r: Runnable) -> Tuple[int, int, int]:
    c = r.candidate
    if c.phase == "prefill":
        inflight = c.prefill_group_leased_members + c.prefill_group_active_members
        if inflight == 0:
            return (1, 0, 0)
        return (0, max(0, c.prefill_group_total_members - inflight), (1 << 32) - 1 - inflight)
    return (2, 0, 0)


def runtime_mode_priority(mode: str) -> int:
    return {"latency_first": 0, "resilient_edge": 1, "throughput_first": 2, "fit_first": 3}[mode]


def topology_rank(mode: str, r: Runnable) -> int:
    if r.candidate.phase != "decode":
        return 0
    return r.candidate.decode_topology_rank if mode == "throughput_first" else 0


def decode_group_order_time(r: Runnable) -> str:
    c = r.candidate
    if c.phase == "decode" and c.decode_cohort_oldest_ready_at is not None:
        return c.decode_cohort_oldest_ready_at
    return r.ready_at


def _session_lease_rank(r: Runnable) -> str:
    if r.candidate.phase != "decode":
        return "z"
    return {"leased": "a", "ready": "b", "active": "c"}.get(r.candidate.decode_queue_status or "", "z")


def decode_session_order_time(r: Runnable) -> str:
    if r.candidate.phase == "decode":
        return f"{_session_lease_rank(r)}:{r.ready_at}"
    return r.candidate.assigned_at


def _cohort_fill_target(c: Candidate) -> Tuple[int, int]:
    fill = c.decode_cohort_leased_sessions + c.decode_cohort_active_sessions
    target = c.decode_lease_target_session_count
    return fill, (target if target is not None else max(fill, 1))


def owned_cohort_age_order(r: Runnable, mode: str) -> str:
    c = r.candidate
    if c.phase != "decode":
        return FAR_FUTURE
    owned = c.group_lease_owner_device_id is not None
    if mode != "latency_first" and not owned and c.decode_cohort_oldest_ready_at is not None:
        return decode_group_order_time(r)
    if owned:
        fill, target = _cohort_fill_target(c)
        if fill < target:
            return decode_group_order_time(r)
    return FAR_FUTURE


def decode_group_fill_rank(mode: str, r: Runnable) -> int:
    c = r.candidate
    if c.phase != "decode":
        return 0
    if c.group_lease_owner_device_id is None:
        ready = min(max(c.decode_cohort_ready_sessions, 1), 31)
        blocked = min(c.decode_cohort_blocked_sessions, 31)
        target = min(c.decode_lease_target_session_count if c.decode_lease_target_session_count is not None else 1, 31)
        if mode == "fit_first":
            fresh = ((31 - target) << 10) + ((31 - blocked) << 5) + ready
        elif mode == "throughput_first":
            fresh = (target << 10) + (ready << 5) + (31 - blocked)
        elif mode == "resilient_edge":
            fresh = ((31 - blocked) << 10) + ((31 - target) << 5) + ready
        else:
            fresh = (ready << 10) + ((31 - blocked) << 5) + target
        return 1_999_999 - fresh
    fill, target = _cohort_fill_target(c)
    if fill >= target:
        return 2_000_000
    remaining = max(0, target - fill)
    rem_rank = min(remaining, 31) if mode in ("fit_first", "resilient_edge") else 31 - min(remaining, 31)
    density = min(fill, 31) if mode == "fit_first" else 31 - min(fill, 31)
    ready_rank = 31 - min(c.decode_cohort_ready_sessions, 31)
    blocked_rank = min(c.decode_cohort_blocked_sessions, 31)
    if mode == "throughput_first":
        keys = (density, ready_rank, blocked_rank, rem_rank)
    elif mode == "fit_first":
        keys = (rem_rank, density, blocked_rank, ready_rank)
    elif mode == "resilient_edge":
        keys = (blocked_rank, rem_rank, density, ready_rank)
    else:
        keys = (rem_rank, density, ready_rank, blocked_rank)
    return (keys[0] << 15) + (keys[1] << 10) + (keys[2] << 5) + keys[3]


def _throughput_priority(r: Runnable) -> int:
    c = r.candidate
    if c.phase != "decode":
        return 2
    return 0 if (c.group_lease_owner_device_id is not None and c.decode_queue_status == "leased") else 1


def _resilient_priority(r: Runnable) -> int:
    return {"prefill_member": 0, "decode_ready": 0, "prefill_leased": 1, "decode_member": 1,
            "decode_leased": 2}.get(r.candidate.group_status, 3)


def mode_rank(mode: str, r: Runnable, submitter_leased: int, job_leased: int) -> tuple:
    c = r.candidate
    decode_bias = int(c.phase != "decode")
    prefill_bias = int(c.phase != "prefill")
    fill = decode_group_fill_rank(mode, r)
    age = owned_cohort_age_order(r, mode)
    order_time = decode_group_order_time(r)
    if mode == "fit_first":
        return (prefill_bias, fill, decode_bias, age, submitter_leased, job_leased, c.created_at)
    if mode == "throughput_first":
        return (_throughput_priority(r), fill, 0, age, job_leased, submitter_leased, order_time)
    if mode == "latency_first":
        return (decode_bias, fill, 0, age, submitter_leased, job_leased, order_time)
    return (_resilient_priority(r), fill, int(c.group_status not in ("decode_ready", "prefill_member")), age,
            submitter_leased + job_leased, 0, order_time)


def rank_candidate(r: Runnable, mode: str, pol: SchedulingPolicy, model_soft_cap: int, capacity_soft_cap: int,
                   snap: Snapshot) -> tuple:
    c = r.candidate
    coord = coordination_rank(r)
    fairness = (int(snap.active_jobs_by_submitter.get(c.submitted_by_device_id, 0) >= pol.submitter_active_job_soft_cap),
                int(snap.active_jobs_by_model.get(c.model_id, 0) >= model_soft_cap),
                int(snap.active_capacity_by_model.get(c.model_id, 0) >= capacity_soft_cap))
    pr = mode_rank(mode, r, snap.leased_assignments_by_submitter.get(c.submitted_by_device_id, 0),
                   snap.leased_assignments_by_job.get(c.job_id, 0))
    session_key = f"{decode_session_order_time(r)}:{c.assignment_id}"
    return coord + fairness + (runtime_mode_priority(c.runtime_mode),) + pr[:3] + \
        ((pr[3], pr[4], pr[5], pr[6], session_key, topology_rank(mode, r)),)


def schedule(candidates: Sequence[Candidate], requesting_device_id: str, now: str, mode: str = "fit_first",
             pol: Optional[SchedulingPolicy] = None, snap: Optional[Snapshot] = None) -> Decision:
    """Classify every candidate, then pick the runnable one with the smallest rank."""
    if mode not in MODES:
        raise ValueError(f"unknown scheduler mode {mode!r}")
    pol = pol or SchedulingPolicy()
    snap = snap or Snapshot()
    runnable, blocked = [], []
    for c in candidates:
        v = classify(c, requesting_device_id, now)
        if isinstance(v, tuple):
            blocked.append(Blocked(c.session_id, c.job_id, c.assignment_id, v[0]))
        else:
            runnable.append(Runnable(c, v))
    if not runnable:
        return Decision(None, blocked)
    model_cap = max(1, snap.online_worker_count // max(1, pol.model_active_job_soft_cap_divisor))
    cap_cap = max(1, snap.online_capacity_units // max(1, pol.capacity_unit_soft_cap_divisor))
    best = min(runnable, key=lambda r: rank_candidate(r, mode, pol, model_cap, cap_cap, snap))
    return Decision(best.candidate.assignment_id, blocked)


def select_claim(candidates: Sequence[Candidate], requesting_device_id: str, now: str, mode: str = "fit_first",
                 pol: Optional[SchedulingPolicy] = None, snap: Optional[Snapshot] = None,
                 waiting_decode_cohort: Optional[Dict[str, str]] = None) -> Decision:
    """Full claim order: (1) a prefill of a group whose other members are already leased or active,
    oldest job first; (2) a prefill whose decode cohort has ready sessions waiting
    (``waiting_decode_cohort``: assignment id -> oldest ready time of its cohort); (3) ``schedule``."""
    pre = [c for c in candidates if c.phase == "prefill" and c.group_status in ("prefill_member", "prefill_leased")]
    inflight = [c for c in pre if c.prefill_group_leased_members + c.prefill_group_active_members > 0]
    if inflight:
        c = min(inflight, key=lambda c: (c.created_at, c.assignment_id))
        return Decision(c.assignment_id, [])
    if waiting_decode_cohort:
        waiting = [c for c in pre if c.assignment_id in waiting_decode_cohort]
        if waiting:
            c = min(waiting, key=lambda c: (waiting_decode_cohort[c.assignment_id], c.created_at, c.assignment_id))
            return Decision(c.assignment_id, [])
    return schedule(candidates, requesting_device_id, now, mode, pol, snap)
