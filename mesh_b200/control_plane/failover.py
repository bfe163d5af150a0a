"""Failover engine: what happens to a session when some of its workers disappear.

Restates ``control-plane/src/services/failover.rs:98-700`` and its helpers (``:2400-2700``):

* losses outside the active segment's participants leave the session ``healthy``;
* losing a prefill participant fails the session (no regroup mid-prefill; manual intervention);
* losing a decode participant regroups: the refreshed plan's decode group if the planner found one,
  else the smallest set of surviving group members that still covers the active column span
  (survivors alone, then, with ``prefer_replacement``, the original group size, then any size);
  members are tried by capacity, then memory, then ring position;
* the resume mode: ``immediate`` when nobody new joins (a shrink) or every new member already holds
  a completed live KV handoff from the KV owner at least as recent as the session; else
  ``requires_live_kv_transfer`` when the KV owner survives into the new group, is in the plan's
  KV support group with a dataplane address, and every target member is in the recovery support
  group with one; else ``requires_checkpoint_transfer`` -- which fails the session when no
  checkpoint (or no transfer source) exists;
* a regroup that needs a transfer pauses the session (``blocked_on_transfer``); otherwise the
  session is ``resume_ready`` and goes back to ``ready``;
* the next KV owner is the current one if it stays, else the target member with the newest KV,
  then a checkpoint, then the most capacity units; the transfer source is the surviving KV owner,
  else the device that holds the latest checkpoint.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Set, Tuple

from .layout import Member

RECOVERY_STATES = ("healthy", "resume_ready", "paused", "failed")
RESUME_MODES = ("none", "immediate", "requires_live_kv_transfer", "requires_checkpoint_transfer",
                "manual_intervention")


@dataclass
class SessionView:
    session_id: str
    status: str                      # e.g. decode_active, decode_ready, prefill_active
    phase: str                       # phase of the active segment: prefill | decode
    participants: List[str]          # active segment participants
    kv_owner_device_id: str
    kv_sequence_position: int = 0
    latest_checkpoint_device_id: Optional[str] = None
    latest_checkpoint_created_at: Optional[str] = None
    segment_id: str = ""


@dataclass
class KvTransfer:
    segment_id: str
    source_device_id: str
    target_device_id: str
    transfer_kind: str               # live_kv_handoff | checkpoint
    status: str
    kv_sequence_position: int = 0


@dataclass
class SupportGroups:
    """Members of the plan's KV and recovery support groups."""
    kv: Set[str] = field(default_factory=set)
    recovery: Set[str] = field(default_factory=set)


@dataclass
class Decision:
    recovery_state: str
    strategy: str                    # none | replace | shrink | fail
    resume_mode: str
    reason: str
    lost_device_ids: List[str] = field(default_factory=list)
    replacement_device_ids: List[str] = field(default_factory=list)
    target_participant_device_ids: List[str] = field(default_factory=list)
    next_kv_owner_device_id: Optional[str] = None
    transfer_source_device_id: Optional[str] = None
    pause_required: bool = False
    session_status: Optional[str] = None
    decode_queue_status: Optional[str] = None   # status the queue entry gets now
    clear_lease: bool = False

    def to_json(self) -> dict:
        return dict(self.__dict__)


# ---------------------------------------------------------------------------------------------- coverage
def coverage_target(participants: Sequence[str], members: Dict[str, Member]) -> Tuple[int, int]:
    missing = [d for d in participants if d not in members]
    if missing:
        raise ValueError(f"execution group is missing participant {missing[0]}")
    if not participants:
        raise ValueError("no active participants available")
    return (min(members[d].column_start for d in participants), max(members[d].column_end for d in participants))


def covers_required_span(members: Dict[str, Member], selected: Sequence[str], span: Tuple[int, int]) -> bool:
    ranges = sorted((members[d].column_start, members[d].column_end) for d in selected if d in members)
    if not ranges or ranges[0][0] > span[0]:
        return False
    end = ranges[0][1]
    for a, b in ranges[1:]:
        if a > end:
            return False
        end = max(end, b)
    return end >= span[1]


def _ring_order(members: Dict[str, Member], ids: Sequence[str]) -> List[str]:
    return sorted(ids, key=lambda d: (members[d].ring_position if d in members else 1 << 31, d))


def find_covering_set(available: Sequence[Member], required: Sequence[str], span: Tuple[int, int],
                      preferred_size: Optional[int]) -> Optional[List[str]]:
    """Smallest set (from ``preferred_size``, or the required count, upwards) holding every required
    device plus extra members, tried in capacity / memory / ring order, whose spans cover ``span``."""
    by_id = {m.device_id: m for m in available}
    req = list(required)
    pool = sorted((m for m in available if m.device_id not in set(req)),
                  key=lambda m: (-m.assigned_capacity_units, -m.contributed_memory, m.ring_position))
    lo = max(preferred_size if preferred_size is not None else len(req), len(req))
    hi = min(max(preferred_size if preferred_size is not None else len(available), len(req)), len(available))

    def choose(k, start, cur):
        if k == 0:
            return list(cur) if covers_required_span(by_id, cur, span) else None
        for i in range(start, len(pool) - k + 1):
            cur.append(pool[i].device_id)
            got = choose(k - 1, i + 1, cur)
            cur.pop()
            if got is not None:
                return got
        return None

    for size in range(lo, hi + 1):
        extra = size - len(req)
        if extra > len(pool):
            continue
        got = choose(extra, 0, list(req))
        if got is not None:
            return _ring_order(by_id, got)
    return None


# ---------------------------------------------------------------------------------------------- transfers
def select_transfer_source(s: SessionView, lost: Set[str], target: Sequence[str]) -> Optional[str]:
    if s.kv_owner_device_id in target and s.kv_owner_device_id not in lost:
        return s.kv_owner_device_id
    return s.latest_checkpoint_device_id


def live_kv_resume_ready(s: SessionView, active: Set[str], target: Sequence[str], introduced: Sequence[str],
                         lost: Set[str], transfers: Sequence[KvTransfer]) -> bool:
    owner = s.kv_owner_device_id
    if not introduced or owner not in active or owner not in target or owner in lost:
        return False
    return all(any(t.segment_id == s.segment_id and t.source_device_id == owner and t.target_device_id == d and
                   t.transfer_kind == "live_kv_handoff" and t.status == "completed" and
                   t.kv_sequence_position >= s.kv_sequence_position for t in transfers) for d in introduced)


def live_kv_transfer_possible(s: SessionView, active: Set[str], target: Sequence[str], lost: Set[str],
                              support: Optional[SupportGroups], dataplane: Dict[str, bool]) -> bool:
    owner = s.kv_owner_device_id
    if owner not in active or owner not in target or owner in lost or support is None:
        return False
    if not support.kv or not support.recovery:
        return False
    return (owner in support.kv and dataplane.get(owner, False) and
            all(d in support.recovery and dataplane.get(d, False) for d in target))


def select_next_kv_owner(target: Sequence[str], s: SessionView, kv_positions: Dict[str, int],
                         members: Dict[str, Member]) -> str:
    if s.kv_owner_device_id in target:
        return s.kv_owner_device_id
    if not target:
        raise ValueError(f"session {s.session_id} has no surviving participant to own KV state")
    has_ckpt = int(s.latest_checkpoint_created_at is not None)
    return max(target, key=lambda d: (kv_positions.get(d, 0), has_ckpt,
                                      members[d].assigned_capacity_units if d in members else 0))


# ---------------------------------------------------------------------------------------------- engine
class FailoverEngine:
    def __init__(self, prefer_replacement: bool = True):
        self.prefer_replacement = prefer_replacement

    @staticmethod
    def _failed(s: SessionView, lost: Sequence[str], detail: str) -> Decision:
        return Decision("failed", "fail", "manual_intervention", f"{detail}: {', '.join(lost)}", list(lost),
                        next_kv_owner_device_id=s.kv_owner_device_id, pause_required=True, session_status="failed",
                        decode_queue_status="failed", clear_lease=True)

    def evaluate(self, s: SessionView, group: Sequence[Member], lost_device_ids: Sequence[str],
                 decode_queue_status: Optional[str] = None, transfers: Sequence[KvTransfer] = (),
                 refreshed_target: Optional[Tuple[List[str], str]] = None,
                 support: Optional[SupportGroups] = None, member_status: Optional[Dict[str, str]] = None,
                 kv_positions: Optional[Dict[str, int]] = None) -> Decision:
        """``group``: members of the active execution group; ``refreshed_target``: (participants,
        kv owner) of a decode group the planner re-formed on the live topology, if any;
        ``member_status``: serving-group record status per device (superseded / failed members are
        not candidates)."""
        lost = set(lost_device_ids)
        lost_active = sorted(d for d in s.participants if d in lost)
        if not lost_active:
            return Decision("healthy", "none", "none", "No active participant loss detected",
                            target_participant_device_ids=list(s.participants))
        if s.phase == "prefill":
            return Decision("failed", "fail", "manual_intervention",
                            f"Prefill participant loss ({', '.join(lost_active)}) cannot safely regroup without "
                            f"replaying the session", lost_active, next_kv_owner_device_id=s.kv_owner_device_id,
                            pause_required=True, session_status="failed", decode_queue_status="failed",
                            clear_lease=True)
        members = {m.device_id: m for m in group}
        status = member_status or {}
        survivors = [d for d in s.participants if d not in lost]
        span = coverage_target(s.participants, members)
        available = [m for m in group if m.device_id not in lost and status.get(m.device_id) not in
                     ("superseded", "failed")]
        if refreshed_target is not None:
            target, next_owner = list(refreshed_target[0]), refreshed_target[1]
        else:
            target = find_covering_set(available, survivors, span, len(survivors))
            if target is None and self.prefer_replacement:
                target = find_covering_set(available, survivors, span, len(s.participants))
            if target is None:
                target = find_covering_set(available, survivors, span, None)
            if target is None:
                return self._failed(s, lost_active, "Remaining decode members can no longer cover the active "
                                                    "shard span")
            next_owner = select_next_kv_owner(target, s, kv_positions or {}, members)
        introduced = [d for d in target if d not in s.participants]
        source = select_transfer_source(s, lost, target)
        active = set(s.participants)
        live_ready = live_kv_resume_ready(s, active, target, introduced, lost, transfers)
        dataplane = {m.device_id: any(a.startswith("dataplane://") for a in m.listen_addrs) for m in group}
        if not introduced or live_ready:
            mode = "immediate"
        elif live_kv_transfer_possible(s, active, target, lost, support, dataplane):
            mode = "requires_live_kv_transfer"
        else:
            mode = "requires_checkpoint_transfer"
        transfer = mode in ("requires_live_kv_transfer", "requires_checkpoint_transfer")
        if mode == "requires_checkpoint_transfer" and (
                source is None or s.latest_checkpoint_device_id is None or s.latest_checkpoint_created_at is None):
            return self._failed(s, lost_active, "Decode regroup requires checkpoint transfer, but no checkpoint "
                                                "is available")
        strategy = "replace" if introduced else "shrink"
        pause = s.status == "decode_active" or decode_queue_status in ("leased", "active")
        if transfer:
            reason = (f"Decode regroup replaces lost participants ({', '.join(lost_active)}) and pauses until "
                      + ("live KV handoff completes" if mode == "requires_live_kv_transfer"
                         else "checkpoint transfer completes"))
        elif not introduced:
            reason = f"Decode can shrink to surviving participants after losing {', '.join(lost_active)}"
        elif live_ready:
            reason = (f"Decode can replace lost participants ({', '.join(lost_active)}) using a completed live KV "
                      f"handoff contract")
        else:
            reason = f"Decode can replace lost participants ({', '.join(lost_active)}) without blocking on transfer"
        return Decision("paused" if transfer else "resume_ready", strategy, mode, reason, lost_active,
                        introduced, target, next_owner, source, pause or transfer, "decode_ready",
                        "blocked_on_transfer" if transfer else "ready", pause or transfer)
