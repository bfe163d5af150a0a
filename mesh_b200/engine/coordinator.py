"""InferenceCoordinator: the serving API of the engine (the reference's ``zip`` coordinator).

Restated behaviour (``agent/src/inference/coordinator.rs``):

* sessions keyed by session id with runtime status active / paused / evicted (``:601-895``);
* a fair decode queue ordered by (decode steps served, fairness epoch) and a microbatch builder
  that starts from a primary session and admits others within the class, fast-path bucket,
  KV-skew, batch-size and KV-budget guardrails (``:731-760``, ``:992-1250``, ``:1467-1496``) -
  implemented natively in ``mesh_b200._runtime.DecodeScheduler``;
* prefill / decode segments (``:1737-1855``, ``:2075-2418``), checkpoints every
  ``checkpoint_interval`` tokens (``job.rs:322-328``), checkpoint-backed export / hydrate of a
  session (``:1529-1597``, ``:1916-1957``);
* a recovery governor limiting checkpoint restores (5 s cooldown, 8 loads per minute,
  ``:146-183``) and KV-memory-budget eviction of idle sessions (``:897-990``).

Backends: ``GpuBackend`` drives the sm_100a engine (``serving.Engine``); ``CpuReferenceBackend``
runs the fp32 host oracle (the reference's cpu provider restated).
"""
from __future__ import annotations

import time
from collections import deque
from dataclasses import asdict, dataclass, field
from typing import Dict, List, Optional

from ..config import EngineConfig
from .checkpoint import Checkpoint, CheckpointManager
from .stats import InferenceStats
from .types import (DecodeBatchPlan, DecodeBatchSlot, ExecutionPhase, GenerationConfig, InferenceRequest,
                    InferenceResult, InferenceRuntimeMode, PrefillComplete, SessionEvictionReason,
                    SessionPauseReason, SessionRuntimeStatus)


# ------------------------------------------------------------------------------------------------
# scheduler: native when built, else a Python restatement with the same semantics
# ------------------------------------------------------------------------------------------------
class _PyDecodeScheduler:
    def __init__(self):
        self.s: Dict[int, dict] = {}
        self.q: Dict[int, tuple] = {}
        self.epoch = 0

    def register_session(self, sid, class_key=0, kv_tokens=0, token_ceiling=-1, mode=1):
        self.s[sid] = dict(cls=class_key, kv=kv_tokens, ceil=token_ceiling, mode=mode, served=0, queued=False,
                           complete=False)

    def update(self, sid, kv_tokens, token_ceiling=-1):
        self.s[sid]["kv"] = kv_tokens
        self.s[sid]["ceil"] = token_ceiling

    def set_complete(self, sid, c):
        self.s[sid]["complete"] = c

    def served(self, sid):
        self.s[sid]["served"] += 1

    def steps_served(self, sid):
        return self.s[sid]["served"]

    def enqueue(self, sid):
        x = self.s[sid]
        if x["queued"] or x["complete"]:
            return False
        self.epoch += 1
        x["queued"] = True
        self.q[sid] = (x["served"], self.epoch, sid)
        return True

    def remove(self, sid):
        self.q.pop(sid, None)
        if sid in self.s:
            self.s[sid]["queued"] = False

    def drop(self, sid):
        self.remove(sid)
        self.s.pop(sid, None)

    def queued(self):
        return [t[2] for t in sorted(self.q.values())]

    def __len__(self):
        return len(self.q)

    @staticmethod
    def _skew_ok(mode, mn, mx):
        if mn == 0 or mx <= mn:
            return True
        if mode == 1:
            return mx <= max(mn * 2, mn + 512)
        if mode == 2:
            return mx <= max((mn * 3 + 1) // 2, mn + 256)
        return True

    def build_batch(self, primary, max_batch, max_total_kv):
        max_batch, max_total_kv = max(1, max_batch), max(1, max_total_kv)
        slots, deferred, admitted = [], [], []
        total = d_cap = d_kv = d_guard = 0
        bmin = bmax = None
        cls = ceil = None
        mode = 1
        if primary in self.q:
            t = self.q[primary]
            x = self.s[primary]
            if not x["complete"]:
                cls, mode, ceil = x["cls"], x["mode"], x["ceil"]
                slots.append((primary, t[1], x["kv"]))
                bmin = bmax = x["kv"]
                total += x["kv"]
            admitted.append(primary)
        for t in sorted(self.q.values()):
            sid = t[2]
            if sid == primary:
                continue
            x = self.s.get(sid)
            if x is None or x["complete"]:
                admitted.append(sid)
                continue
            if cls is not None:
                if mode in (1, 2) and x["cls"] != cls:
                    d_guard += 1
                    deferred.append((sid, t[1]))
                    continue
            else:
                cls, mode, ceil = x["cls"], x["mode"], x["ceil"]
            if mode in (1, 2) and ceil is not None and ceil >= 0 and x["ceil"] != ceil:
                d_guard += 1
                deferred.append((sid, t[1]))
                continue
            pmin = x["kv"] if bmin is None else min(bmin, x["kv"])
            pmax = x["kv"] if bmax is None else max(bmax, x["kv"])
            if not self._skew_ok(mode, pmin, pmax):
                d_guard += 1
                deferred.append((sid, t[1]))
                continue
            full = len(slots) >= max_batch
            kv_out = bool(slots) and total + x["kv"] > max_total_kv
            if full or kv_out:
                if full:
                    d_cap += 1
                else:
                    d_kv += 1
                deferred.append((sid, t[1]))
                continue
            slots.append((sid, t[1], x["kv"]))
            bmin, bmax = pmin, pmax
            total += x["kv"]
            admitted.append(sid)
        for sid in admitted:
            self.remove(sid)
        return dict(slots=slots, deferred=deferred, total_kv_tokens=total, deferred_for_capacity=d_cap,
                    deferred_for_kv_budget=d_kv, deferred_for_guardrail=d_guard)


def make_scheduler():
    try:
        from .. import _runtime
        return _runtime.DecodeScheduler()
    except ImportError:
        return _PyDecodeScheduler()


# ------------------------------------------------------------------------------------------------
@dataclass
class RecoveryGovernor:
    """Limits checkpoint-backed session loads: a cooldown per session and a per-minute budget."""
    cooldown_s: float = 5.0
    max_loads_per_minute: int = 8
    last_load: Dict[str, float] = field(default_factory=dict)
    loads: deque = field(default_factory=deque)

    def check(self, session_id: str, now: Optional[float] = None) -> Optional[str]:
        now = time.monotonic() if now is None else now
        while self.loads and now - self.loads[0] > 60.0:
            self.loads.popleft()
        t = self.last_load.get(session_id)
        if t is not None and now - t < self.cooldown_s:
            return "cooldown"
        if len(self.loads) >= self.max_loads_per_minute:
            return "budget"
        return None

    def record(self, session_id: str, now: Optional[float] = None):
        now = time.monotonic() if now is None else now
        self.last_load[session_id] = now
        self.loads.append(now)


# ------------------------------------------------------------------------------------------------
@dataclass
class ActiveSession:
    request: InferenceRequest
    handle: int
    generated: List[int] = field(default_factory=list)
    status: SessionRuntimeStatus = SessionRuntimeStatus.ACTIVE
    pause_reason: Optional[SessionPauseReason] = None
    eviction_reason: Optional[SessionEvictionReason] = None
    prefilled: bool = False
    t_start: float = field(default_factory=time.perf_counter)
    ttft_ms: Optional[float] = None
    last_active: float = field(default_factory=time.monotonic)
    recovered: bool = False
    last_checkpoint_token: int = 0

    @property
    def complete(self) -> bool:
        return len(self.generated) >= self.request.config.max_tokens

    @property
    def kv_tokens(self) -> int:
        return len(self.request.prompt_tokens) + max(0, len(self.generated) - 1)


class InferenceCoordinator:
    def __init__(self, backend, config: Optional[EngineConfig] = None,
                 checkpoints: Optional[CheckpointManager] = None, stats: Optional[InferenceStats] = None,
                 worker_id: str = "local", model_id: str = ""):
        self.backend = backend
        self.config = config or EngineConfig()
        self.checkpoints = checkpoints
        self.stats = stats or InferenceStats()
        self.worker_id = worker_id
        self.model_id = model_id
        self.sessions: Dict[str, ActiveSession] = {}
        self.by_handle: Dict[int, str] = {}
        self.sched = make_scheduler()
        self.governor = RecoveryGovernor(self.config.recovery_cooldown_s, self.config.recovery_max_loads_per_minute)
        self._handles = 0
        self.completed: Dict[str, InferenceResult] = {}

    # -------------------------------------------------------------------------------- sessions
    def _new_handle(self) -> int:
        self._handles += 1
        return self._handles

    def submit(self, request: InferenceRequest) -> str:
        if request.session_id in self.sessions:
            raise ValueError(f"session {request.session_id} already active")
        active = [s for s in self.sessions.values() if s.status == SessionRuntimeStatus.ACTIVE]
        if len(active) >= self.config.max_active_sessions:
            self.enforce_memory_budget(force_one=True)
        h = self._new_handle()
        sess = ActiveSession(request=request, handle=h)
        self.sessions[request.session_id] = sess
        self.by_handle[h] = request.session_id
        mode = request.runtime_mode if isinstance(request.runtime_mode, InferenceRuntimeMode) else \
            InferenceRuntimeMode(request.runtime_mode)
        self.sched.register_session(h, self.backend.class_key, len(request.prompt_tokens),
                                    self.backend.token_ceiling(len(request.prompt_tokens)), mode.native)
        return request.session_id

    def _prefill(self, sess: ActiveSession) -> None:
        cfg = sess.request.config
        t0 = time.perf_counter()
        # seeds: job id bits xor token position (the backend applies the position)
        tok = self.backend.prefill(sess.handle, sess.request.prompt_tokens, cfg.temperature, cfg.top_p,
                                   sess.request.seed_for_position(0))
        sess.ttft_ms = (time.perf_counter() - sess.t_start) * 1e3
        sess.generated.append(int(tok))
        sess.prefilled = True
        self.stats.add("total_prompt_tokens", len(sess.request.prompt_tokens))
        self.stats.add("total_tokens_generated", 1)
        self.stats.add("device_prefill_time_ms", (time.perf_counter() - t0) * 1e3)
        self._drain_backend_counters()
        self.sched.update(sess.handle, sess.kv_tokens, self.backend.token_ceiling(sess.kv_tokens))
        if sess.complete:
            self.sched.set_complete(sess.handle, True)
        else:
            self.sched.enqueue(sess.handle)

    def _drain_backend_counters(self) -> None:
        drain = getattr(self.backend, "drain_counters", None)
        if drain is not None:
            for k, v in drain().items():
                self.stats.add(k, v)

    def build_next_decode_batch(self, primary_session: Optional[str] = None) -> DecodeBatchPlan:
        h = self.sessions[primary_session].handle if primary_session in self.sessions else -1
        d = self.sched.build_batch(h, self.config.max_decode_batch_size, self.config.max_decode_batch_kv_tokens)
        plan = DecodeBatchPlan(
            slots=[DecodeBatchSlot(self.by_handle[sid], epoch, kv) for sid, epoch, kv in d["slots"]],
            deferred=[self.by_handle[sid] for sid, _ in d["deferred"]], total_kv_tokens=d["total_kv_tokens"],
            deferred_for_capacity=d["deferred_for_capacity"], deferred_for_kv_budget=d["deferred_for_kv_budget"],
            deferred_for_guardrail=d["deferred_for_guardrail"])
        return plan

    def _decode_microbatch(self, plan: DecodeBatchPlan) -> List[str]:
        sess = [self.sessions[s.session_id] for s in plan.slots]
        if not sess:
            return []
        items = [(s.handle, s.request.config.temperature, s.request.config.top_p,
                  s.request.seed_for_position(0)) for s in sess]
        toks = self.backend.decode(items)
        self._drain_backend_counters()
        st = self.stats
        st.add("decode_microbatches_executed")
        st.add("decode_sessions_batched", len(sess))
        st.add("decode_batch_size_peak", len(sess))
        st.add("decode_batch_kv_tokens_total", plan.total_kv_tokens)
        st.add("decode_batch_deferred_sessions", len(plan.deferred))
        st.add("decode_batch_capacity_deferrals", plan.deferred_for_capacity)
        st.add("decode_batch_kv_budget_deferrals", plan.deferred_for_kv_budget)
        st.add("decode_batch_guardrail_deferrals", plan.deferred_for_guardrail)
        if len(sess) > 1:
            st.add("decode_multi_session_microbatches")
        done = []
        for s, t in zip(sess, toks):
            s.generated.append(int(t))
            s.last_active = time.monotonic()
            st.add("total_tokens_generated", 1)
            self.sched.served(s.handle)
            self.sched.update(s.handle, s.kv_tokens, self.backend.token_ceiling(s.kv_tokens))
            self._maybe_checkpoint(s)
            if s.complete:
                self.sched.set_complete(s.handle, True)
                done.append(s.request.session_id)
            else:
                self.sched.enqueue(s.handle)
        return done

    def step(self) -> List[InferenceResult]:
        """One scheduling step: prefill one waiting session, else one decode microbatch."""
        results = []
        for sess in self.sessions.values():
            if sess.status == SessionRuntimeStatus.ACTIVE and not sess.prefilled:
                self._prefill(sess)
                if sess.complete:
                    results.append(self._finish(sess.request.session_id))
                return results
        plan = self.build_next_decode_batch()
        for sid in self._decode_microbatch(plan):
            results.append(self._finish(sid))
        return results

    def run_until_idle(self, max_steps: int = 1_000_000) -> List[InferenceResult]:
        out = []
        for _ in range(max_steps):
            if not any(s.status == SessionRuntimeStatus.ACTIVE and not s.complete for s in self.sessions.values()):
                break
            out.extend(self.step())
        return out

    def _finish(self, session_id: str) -> InferenceResult:
        s = self.sessions.pop(session_id)
        self.by_handle.pop(s.handle, None)
        self.sched.drop(s.handle)
        self.backend.release(s.handle)
        dt = (time.perf_counter() - s.t_start) * 1e3
        res = InferenceResult(job_id=s.request.job_id, success=True, generated_tokens=list(s.generated),
                              prompt_tokens=len(s.request.prompt_tokens), completion_tokens=len(s.generated),
                              execution_time_ms=int(dt), time_to_first_token_ms=int(s.ttft_ms or 0),
                              tokens_per_second=len(s.generated) / max(dt / 1e3, 1e-9),
                              recovered_from_checkpoint=s.recovered)
        self.stats.add("jobs_completed")
        self.stats.add("total_inference_time_ms", dt)
        self.completed[s.request.job_id] = res
        return res

    # -------------------------------------------------------------------------------- entry points
    def process_inference(self, request: InferenceRequest) -> InferenceResult:
        """Prefill and decode one request to completion (other active sessions keep their place)."""
        sid = self.submit(request)
        try:
            while sid in self.sessions:
                self.step()
        except Exception as e:  # surface as a failed result like the reference
            import traceback
            self.stats.add("jobs_failed")
            e = RuntimeError(f"{e}\n{traceback.format_exc()}")
            if sid in self.sessions:
                s = self.sessions.pop(sid)
                self.sched.drop(s.handle)
                self.backend.release(s.handle)
            return InferenceResult.failure(request.job_id, str(e), len(request.prompt_tokens))
        return self.completed[request.job_id]

    def process_segment(self, request: InferenceRequest):
        """Prefill segment -> PrefillComplete (session stays resident for decode); decode segment ->
        run the session to completion -> InferenceResult."""
        if request.phase == ExecutionPhase.PREFILL:
            sid = self.submit(request)
            s = self.sessions[sid]
            self._prefill(s)
            return PrefillComplete(job_id=request.job_id, session_id=sid, completion_tokens=len(s.generated),
                                   execution_time_ms=int((time.perf_counter() - s.t_start) * 1e3),
                                   time_to_first_token_ms=int(s.ttft_ms or 0), kv_cache_seq_len=s.kv_tokens)
        if request.session_id not in self.sessions:
            raise KeyError(f"Session {request.session_id} is not active for decode scheduling")
        while request.session_id in self.sessions:
            self.step()
        return self.completed[request.job_id]

    # -------------------------------------------------------------------------------- pause / evict
    def pause_session(self, session_id: str, reason: SessionPauseReason) -> None:
        s = self.sessions[session_id]
        s.status = SessionRuntimeStatus.PAUSED
        s.pause_reason = reason
        self.sched.remove(s.handle)

    def resume_session(self, session_id: str) -> None:
        s = self.sessions[session_id]
        if s.status == SessionRuntimeStatus.EVICTED:
            raise RuntimeError("evicted sessions resume from a checkpoint (hydrate_session)")
        s.status = SessionRuntimeStatus.ACTIVE
        s.pause_reason = None
        if s.prefilled and not s.complete:
            self.sched.enqueue(s.handle)

    def evict_session(self, session_id: str, reason: SessionEvictionReason) -> Optional[bytes]:
        """Checkpoint (when possible) and free the session's KV; returns the checkpoint bytes."""
        s = self.sessions[session_id]
        blob = self.export_session_checkpoint_bytes(session_id) if s.prefilled else None
        s.status = SessionRuntimeStatus.EVICTED
        s.eviction_reason = reason
        self.sched.remove(s.handle)
        self.backend.release(s.handle)
        return blob

    def kv_bytes_in_use(self) -> int:
        return sum(self.backend.kv_bytes(s.handle) for s in self.sessions.values()
                   if s.status != SessionRuntimeStatus.EVICTED)

    def enforce_memory_budget(self, force_one: bool = False) -> List[str]:
        """Evict least recently active idle sessions until KV use fits the budget."""
        evicted = []
        cands = sorted((s for s in self.sessions.values() if s.status != SessionRuntimeStatus.EVICTED),
                       key=lambda s: s.last_active)
        for s in cands:
            over = self.kv_bytes_in_use() > self.config.kv_memory_budget_bytes
            if not over and not (force_one and not evicted):
                break
            if s.status == SessionRuntimeStatus.PAUSED or force_one or over:
                self.evict_session(s.request.session_id, SessionEvictionReason.RUNTIME_MEMORY_PRESSURE)
                evicted.append(s.request.session_id)
        return evicted

    # -------------------------------------------------------------------------------- checkpoints
    def _maybe_checkpoint(self, s: ActiveSession) -> None:
        iv = s.request.config.checkpoint_interval
        if self.checkpoints is None or iv <= 0:
            return
        if len(s.generated) - s.last_checkpoint_token >= iv:
            self.checkpoints.save(Checkpoint.from_bytes(self.export_session_checkpoint_bytes(s.request.session_id)))
            s.last_checkpoint_token = len(s.generated)
            self.stats.add("checkpoints_created")

    def export_session_checkpoint_bytes(self, session_id: str) -> bytes:
        s = self.sessions[session_id]
        snap = self.backend.export_kv(s.handle)
        self.stats.add("kv_snapshot_exports")
        self.stats.add("kv_snapshot_export_bytes", len(snap))
        cp = Checkpoint.new(job_id=s.request.job_id, token_index=len(s.generated), request=s.request.to_dict(),
                            generated=s.generated, config=asdict(s.request.config),
                            kv_handoff={"residency": "host_snapshot", "owner_worker_id": self.worker_id,
                                        "source_worker_id": self.worker_id, "payload": snap},
                            model_id=self.model_id, worker_id=self.worker_id)
        return cp.to_bytes()

    def hydrate_session(self, blob: bytes) -> str:
        """Resume a session from checkpoint bytes (its KV restored, decode continues)."""
        cp = Checkpoint.from_bytes(blob)
        req = InferenceRequest.from_dict(cp.request)
        why = self.governor.check(req.session_id)
        if why == "cooldown":
            self.stats.add("recovery_cooldown_rejections")
            raise RuntimeError("recovery cooldown active for session")
        if why == "budget":
            self.stats.add("recovery_budget_rejections")
            raise RuntimeError("recovery budget exhausted")
        self.governor.record(req.session_id)
        self.stats.add("recovery_attempts")
        if req.session_id in self.sessions:
            old = self.sessions.pop(req.session_id)
            self.by_handle.pop(old.handle, None)
            self.sched.drop(old.handle)
        h = self._new_handle()
        payload = (cp.kv_handoff or {}).get("payload")
        if payload is None:
            self.stats.add("recovery_checkpoint_misses")
            raise RuntimeError("checkpoint carries no KV payload")
        self.backend.import_kv(h, payload, req.prompt_tokens, cp.generated_tokens)
        s = ActiveSession(request=req, handle=h, generated=list(cp.generated_tokens), prefilled=True, recovered=True,
                          last_checkpoint_token=len(cp.generated_tokens))
        self.sessions[req.session_id] = s
        self.by_handle[h] = req.session_id
        self.sched.register_session(h, self.backend.class_key, s.kv_tokens, self.backend.token_ceiling(s.kv_tokens),
                                    req.runtime_mode.native)
        if not s.complete:
            self.sched.enqueue(h)
        self.stats.add("checkpoint_recoveries")
        return req.session_id
