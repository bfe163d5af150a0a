"""Control-plane services (business logic behind the HTTP API).

Behaviour restated from the reference control plane (``control-plane/src``):

* device registration and heartbeat (``services/device_service.rs``, ``api/routes.rs``);
* ring topology: sequential positions, weighted GQA-aligned column ranges, neighbours, version
  counter, handoffs and callbacks (``services/ring_manager.rs:140-1091``,
  ``services/topology_notifier.rs``);
* execution planning: prefill and decode execution groups over the ring's TP members, segments
  ``segment-<session>-prefill/-decode``, co-located KV (``services/planner.rs:49-372``);
* submit: tokenize, quote + reserve credits, persist job / session / groups / assignments and a
  decode queue entry ``blocked_on_prefill`` in one transaction (``api/inference.rs:383-765``);
* claim: in-flight prefill assignments first, then decode cohorts for ready sessions, 60 s leases
  (``api/inference.rs:4567-4925``, ``services/scheduler.rs:119-197``); renew / release leases;
* progress: PrefillComplete moves the queue entry to ``ready`` (co-located) or
  ``blocked_on_transfer`` (handoff) (``api/inference.rs:5782-6412``);
* result: completion, settlement through the credit policy, ledger events (``:5320-5781``);
* failover: prefill loss -> fail and release credits; decode loss -> replace with an idle ring
  member, shrink to the survivors when they still cover every column, else fail; resume mode
  from the available checkpoint (``services/failover.rs:174-700``);
* presence: devices silent for 15 s become stale and trigger failover
  (``services/presence.rs:12-96``).
"""
from __future__ import annotations

import hashlib
import json
import os
import time
import uuid
from typing import Dict, List, Optional, Tuple

from ..config import ModelConfig, PRESETS
from . import policy
from .db import Database, dumps, loads

ASSIGNMENT_LEASE_SECS = 60.0
DECODE_QUEUE_STATUSES = ("blocked_on_prefill", "blocked_on_transfer", "ready", "leased", "active", "completed",
                         "failed")


class ApiError(Exception):
    status = 400

    def __init__(self, msg: str, status: int = 400):
        super().__init__(msg)
        self.status = status


class NotFound(ApiError):
    def __init__(self, msg):
        super().__init__(msg, 404)


class Conflict(ApiError):
    def __init__(self, msg):
        super().__init__(msg, 409)


def _now() -> float:
    return time.time()


def _uid() -> str:
    return str(uuid.uuid4())


class ControlPlane:
    def __init__(self, db: Optional[Database] = None, model_store: Optional[str] = None):
        self.db = db or Database()
        self.model_store = model_store
        self.stale_timeout_s = float(os.environ.get("MESHNET_PRESENCE_STALE_TIMEOUT_MS", "15000")) / 1000.0

    # ------------------------------------------------------------------------------------ models
    def model_config(self, model_id: str) -> Tuple[ModelConfig, int]:
        """Attention geometry and total bytes of a model: ``model.json`` in the model store, else a
        built-in preset of the same name."""
        if self.model_store:
            p = os.path.join(self.model_store, model_id, "model.json")
            if os.path.exists(p):
                m = json.load(open(p))
                hd = m["tensor_parallelism_dim"]
                cfg = ModelConfig(hd, m["attention_head_count"], m["kv_head_count"], m.get("num_layers", 1),
                                  m.get("vocab_size", 32000), m.get("intermediate_size", 4 * hd), name=model_id)
                return cfg, int(m.get("total_model_bytes", cfg.param_count() * 2))
        if model_id in PRESETS:
            cfg = PRESETS[model_id]
            return cfg, cfg.param_count() * 2
        raise NotFound(f"unknown model {model_id}")

    def tokenize(self, model_id: str, prompt: str) -> List[int]:
        """Tokenizer of the model store when present (``model_assets.rs:871-891``), else UTF-8 bytes."""
        if self.model_store:
            p = os.path.join(self.model_store, model_id, "tokenizer.json")
            if os.path.exists(p):
                from tokenizers import Tokenizer
                return Tokenizer.from_file(p).encode(prompt).ids
        return list(prompt.encode("utf-8")) or [0]

    # ------------------------------------------------------------------------------------ networks
    def create_network(self, name: str, owner_device_id: Optional[str] = None, scheduling_policy: dict = None) -> dict:
        nid = _uid()
        pol = {"submitter_soft_cap": 1, "model_capacity_divisor": 2, "capacity_divisor": 2,
               "tier_capacity_units": policy.TIER_CAPACITY_UNITS}
        pol.update(scheduling_policy or {})
        with self.db.tx() as c:
            c.execute("INSERT INTO networks VALUES (?,?,?,?,?,?)", (nid, name, owner_device_id, _now(), dumps(pol), "{}"))
        return {"network_id": nid, "name": name, "scheduling_policy": pol}

    def list_networks(self) -> List[dict]:
        return self.db.query("SELECT network_id, name, owner_device_id, created_at FROM networks ORDER BY created_at")

    # ------------------------------------------------------------------------------------ devices
    def register_device(self, device_id: str, network_id: Optional[str], name: str = "", tier: str = "tier2",
                        provider: str = "cpu", contributed_memory: int = 0, capabilities: dict = None,
                        public_key: str = "", certificate: str = "", tensor_plane_addr: str = "") -> dict:
        with self.db.tx() as c:
            c.execute("""INSERT INTO devices (device_id, network_id, name, public_key, certificate, tier, provider,
                         contributed_memory, status, last_heartbeat, created_at, capabilities, tensor_plane_addr)
                         VALUES (?,?,?,?,?,?,?,?,'online',?,?,?,?)
                         ON CONFLICT(device_id) DO UPDATE SET network_id=excluded.network_id, name=excluded.name,
                         tier=excluded.tier, provider=excluded.provider,
                         contributed_memory=excluded.contributed_memory, status='online',
                         last_heartbeat=excluded.last_heartbeat, capabilities=excluded.capabilities,
                         tensor_plane_addr=excluded.tensor_plane_addr""",
                      (device_id, network_id, name, public_key, certificate, tier, provider, contributed_memory,
                       _now(), _now(), dumps(capabilities or {}), tensor_plane_addr))
        return {"device_id": device_id, "status": "online"}

    def heartbeat(self, device_id: str, throughput_tps: Optional[float] = None) -> dict:
        with self.db.tx() as c:
            cur = c.execute("UPDATE devices SET last_heartbeat=?, status='online', throughput_tps=COALESCE(?, "
                            "throughput_tps) WHERE device_id=?", (_now(), throughput_tps, device_id))
            if cur.rowcount == 0:
                raise NotFound(f"device {device_id} not registered")
        return {"device_id": device_id, "status": "online"}

    # ------------------------------------------------------------------------------------ ring
    def _recompute_ring(self, c, network_id: str, model_id: str) -> None:
        cfg, _ = self.model_config(model_id)
        members = [dict(r) for r in c.execute(
            "SELECT m.device_id, m.contributed_memory, d.tier, d.throughput_tps FROM ring_members m "
            "LEFT JOIN devices d ON d.device_id=m.device_id WHERE m.network_id=? AND m.model_id=? "
            "AND m.status='active' ORDER BY m.position", (network_id, model_id)).fetchall()]
        if not members:
            return
        weights = [policy.capacity_weight(policy.CapacityProfile(tier=m["tier"] or "tier2",
                                                                 contributed_memory=m["contributed_memory"] or 0))
                   for m in members]
        ranges = policy.weighted_group_ranges(cfg.hidden_dim, cfg.q_group_width, weights)
        for pos, (m, (a, b)) in enumerate(zip(members, ranges)):
            c.execute("UPDATE ring_members SET position=?, column_start=?, column_end=? WHERE device_id=?",
                      (pos, a, b, m["device_id"]))
        c.execute("INSERT INTO ring_state VALUES (?,?,1,?) ON CONFLICT(network_id, model_id) DO UPDATE SET "
                  "version=version+1, updated_at=excluded.updated_at", (network_id, model_id, _now()))

    def join_ring(self, device_id: str, network_id: str, model_id: str, contributed_memory: int = 0) -> dict:
        dev = self.db.one("SELECT * FROM devices WHERE device_id=?", (device_id,))
        if dev is None:
            raise NotFound(f"device {device_id} not registered")
        self.model_config(model_id)
        with self.db.tx() as c:
            n = c.execute("SELECT COUNT(*) FROM ring_members WHERE network_id=? AND model_id=?",
                          (network_id, model_id)).fetchone()[0]
            c.execute("INSERT INTO ring_members VALUES (?,?,?,?,0,0,?,'active',?) ON CONFLICT(device_id) DO UPDATE "
                      "SET status='active', network_id=excluded.network_id, model_id=excluded.model_id, "
                      "contributed_memory=excluded.contributed_memory",
                      (device_id, network_id, model_id, n, contributed_memory, _now()))
            self._recompute_ring(c, network_id, model_id)
        return self.topology(network_id, model_id)

    def leave_ring(self, device_id: str) -> dict:
        m = self.db.one("SELECT * FROM ring_members WHERE device_id=?", (device_id,))
        if m is None:
            raise NotFound(f"device {device_id} is not a ring member")
        with self.db.tx() as c:
            c.execute("DELETE FROM ring_members WHERE device_id=?", (device_id,))
            self._recompute_ring(c, m["network_id"], m["model_id"])
        return self.topology(m["network_id"], m["model_id"])

    def topology(self, network_id: str, model_id: Optional[str] = None) -> dict:
        args = [network_id]
        q = "SELECT * FROM ring_members WHERE network_id=? AND status='active'"
        if model_id:
            q += " AND model_id=?"
            args.append(model_id)
        members = self.db.query(q + " ORDER BY position", args)
        n = len(members)
        out = []
        for i, m in enumerate(members):
            d = self.db.one("SELECT status, tensor_plane_addr, provider FROM devices WHERE device_id=?",
                            (m["device_id"],)) or {}
            out.append({"device_id": m["device_id"], "position": m["position"], "column_start": m["column_start"],
                        "column_end": m["column_end"], "left_neighbor": members[(i - 1) % n]["device_id"],
                        "right_neighbor": members[(i + 1) % n]["device_id"], "status": d.get("status"),
                        "tensor_plane_addr": d.get("tensor_plane_addr"), "provider": d.get("provider")})
        st = None
        if model_id:
            st = self.db.one("SELECT version FROM ring_state WHERE network_id=? AND model_id=?", (network_id, model_id))
        total = 0
        stable = False
        if model_id and members:
            cfg, _ = self.model_config(model_id)
            total = cfg.hidden_dim
            stable = members[-1]["column_end"] == total and members[0]["column_start"] == 0 and all(
                out[i]["status"] == "online" for i in range(n))
        return {"network_id": network_id, "model_id": model_id, "version": (st or {}).get("version", 0),
                "total_workers": n, "total_columns": total, "stable": stable, "workers": out}

    def check_topology_version(self, network_id: str, model_id: str, version: int) -> dict:
        cur = self.topology(network_id, model_id)["version"]
        return {"current_version": cur, "changed": cur != version}

    def create_handoff(self, network_id, model_id, from_device_id, to_device_id, column_start, column_end) -> dict:
        hid = _uid()
        with self.db.tx() as c:
            c.execute("INSERT INTO ring_handoffs VALUES (?,?,?,?,?,?,?,'pending',?,?)",
                      (hid, network_id, model_id, from_device_id, to_device_id, column_start, column_end, _now(),
                       _now()))
        return self.get_handoff(hid)

    def get_handoff(self, hid: str) -> dict:
        h = self.db.one("SELECT * FROM ring_handoffs WHERE handoff_id=?", (hid,))
        if h is None:
            raise NotFound(f"handoff {hid}")
        return h

    def update_handoff(self, hid: str, status: str) -> dict:
        if status not in ("pending", "in_progress", "completed", "failed", "cancelled"):
            raise ApiError(f"invalid handoff status {status}")
        with self.db.tx() as c:
            c.execute("UPDATE ring_handoffs SET status=?, updated_at=? WHERE handoff_id=?", (status, _now(), hid))
        return self.get_handoff(hid)

    def list_handoffs(self, network_id: Optional[str] = None) -> List[dict]:
        if network_id:
            return self.db.query("SELECT * FROM ring_handoffs WHERE network_id=? ORDER BY created_at", (network_id,))
        return self.db.query("SELECT * FROM ring_handoffs ORDER BY created_at")

    def register_callback(self, device_id: str, url: str) -> dict:
        with self.db.tx() as c:
            c.execute("INSERT INTO ring_callbacks VALUES (?,?,?) ON CONFLICT(device_id) DO UPDATE SET url=excluded.url",
                      (device_id, url, _now()))
        return {"device_id": device_id, "url": url}

    def unregister_callback(self, device_id: str) -> dict:
        with self.db.tx() as c:
            c.execute("DELETE FROM ring_callbacks WHERE device_id=?", (device_id,))
        return {"device_id": device_id, "removed": True}

    # ------------------------------------------------------------------------------------ ledger
    def _ledger(self, c, network_id, device_id, job_id, event_type, credits, details=None):
        c.execute("INSERT INTO ledger_events VALUES (?,?,?,?,?,?,?,?)",
                  (_uid(), network_id, device_id, job_id, event_type, float(credits), dumps(details or {}), _now()))

    def create_ledger_event(self, network_id, device_id, event_type, credits=0.0, job_id=None, details=None) -> dict:
        with self.db.tx() as c:
            self._ledger(c, network_id, device_id, job_id, event_type, credits, details)
        return {"ok": True}

    def list_ledger_events(self, network_id: Optional[str] = None, device_id: Optional[str] = None,
                           limit: int = 100) -> List[dict]:
        q, a = "SELECT * FROM ledger_events WHERE 1=1", []
        if network_id:
            q += " AND network_id=?"
            a.append(network_id)
        if device_id:
            q += " AND device_id=?"
            a.append(device_id)
        rows = self.db.query(q + " ORDER BY created_at DESC LIMIT ?", a + [limit])
        for r in rows:
            r["details"] = loads(r["details"], {})
        return rows

    def ledger_summary(self, network_id: Optional[str] = None) -> dict:
        rows = self.list_ledger_events(network_id, limit=1_000_000)
        earned, spent, reserved = {}, {}, 0.0
        for r in rows:
            if r["event_type"] == "credits_earned":
                earned[r["device_id"]] = earned.get(r["device_id"], 0.0) + r["credits"]
            elif r["event_type"] == "credits_spent":
                spent[r["device_id"]] = spent.get(r["device_id"], 0.0) + r["credits"]
            elif r["event_type"] == "credits_reserved":
                reserved += r["credits"]
            elif r["event_type"] == "credits_released":
                reserved -= r["credits"]
        return {"earned": earned, "spent": spent, "outstanding_reserved": reserved, "events": len(rows)}

    # ------------------------------------------------------------------------------------ inference
    def plan(self, network_id: str, model_id: str, session_id: str) -> dict:
        topo = self.topology(network_id, model_id)
        if not topo["stable"]:
            raise Conflict("ring is not stable: no full column coverage by online workers")
        members = [{"device_id": w["device_id"], "worker_position": w["position"], "total_workers": topo["total_workers"],
                    "shard_column_start": w["column_start"], "shard_column_end": w["column_end"]}
                   for w in topo["workers"]]
        pid = _uid()
        groups = [{"group_id": f"group-{pid}-prefill", "phase": "prefill", "members": members},
                  {"group_id": f"group-{pid}-decode", "phase": "decode", "members": members}]
        segs = [{"segment_id": f"segment-{session_id}-prefill", "phase": "prefill",
                 "execution_group_id": groups[0]["group_id"], "session_id": session_id,
                 "participant_device_ids": [m["device_id"] for m in members]},
                {"segment_id": f"segment-{session_id}-decode", "phase": "decode",
                 "execution_group_id": groups[1]["group_id"], "session_id": session_id,
                 "participant_device_ids": [m["device_id"] for m in members]}]
        return {"plan_id": pid, "model_id": model_id, "execution_groups": groups, "segments": segs,
                "kv_owner_device_id": members[0]["device_id"], "kv_transfer_policy": "co_located",
                "topology_version": topo["version"]}

    def submit_inference(self, network_id: str, model_id: str, prompt: Optional[str] = None,
                         prompt_tokens: Optional[List[int]] = None, max_tokens: int = 100, temperature: float = 0.7,
                         top_p: float = 0.9, submitter_device_id: Optional[str] = None,
                         runtime_mode: str = "throughput_first") -> dict:
        if prompt_tokens is None:
            if prompt is None:
                raise ApiError("prompt or prompt_tokens required")
            prompt_tokens = self.tokenize(model_id, prompt)
        if not prompt_tokens:
            raise ApiError("empty prompt")
        cfg, total_bytes = self.model_config(model_id)
        job_id, session_id = _uid(), _uid()
        plan = self.plan(network_id, model_id, session_id)
        quote = policy.consumption(len(prompt_tokens), max_tokens, total_bytes)
        now = _now()
        with self.db.tx() as c:
            c.execute("""INSERT INTO inference_jobs (job_id, network_id, model_id, submitter_device_id, prompt_tokens,
                         max_tokens, temperature, top_p, status, created_at, updated_at, plan, credits_reserved,
                         runtime_mode) VALUES (?,?,?,?,?,?,?,?,'pending',?,?,?,?,?)""",
                      (job_id, network_id, model_id, submitter_device_id, dumps(prompt_tokens), max_tokens, temperature,
                       top_p, now, now, dumps(plan), quote["total_credits"], runtime_mode))
            c.execute("INSERT INTO inference_sessions VALUES (?,?,'planned','prefill',?,0,?,?)",
                      (session_id, job_id, plan["kv_owner_device_id"], now, now))
            for g in plan["execution_groups"]:
                c.execute("INSERT INTO inference_serving_groups VALUES (?,?,?,?,?,'planned')",
                          (g["group_id"], job_id, session_id, g["phase"], dumps([m["device_id"] for m in g["members"]])))
            for m in plan["execution_groups"][0]["members"]:
                c.execute("""INSERT INTO inference_job_assignments (assignment_id, job_id, session_id, device_id, phase,
                             segment_id, group_id, status, shard_column_start, shard_column_end, worker_position,
                             total_workers, created_at, updated_at) VALUES (?,?,?,?,'prefill',?,?,'pending',?,?,?,?,?,?)""",
                          (_uid(), job_id, session_id, m["device_id"], plan["segments"][0]["segment_id"],
                           plan["execution_groups"][0]["group_id"], m["shard_column_start"], m["shard_column_end"],
                           m["worker_position"], m["total_workers"], now, now))
            c.execute("INSERT INTO inference_decode_queue VALUES (?,?,?,'blocked_on_prefill',NULL,NULL,NULL,0,0,0,?)",
                      (session_id, job_id, network_id, now))
            self._ledger(c, network_id, submitter_device_id, job_id, "credits_reserved", quote["total_credits"], quote)
            self._ledger(c, network_id, submitter_device_id, job_id, "job_started", 0.0, {"model_id": model_id})
            c.execute("INSERT INTO inference_scheduler_events (network_id, job_id, event, details, created_at) "
                      "VALUES (?,?,?,?,?)", (network_id, job_id, "submitted", dumps({"session_id": session_id}), now))
        return {"job_id": job_id, "session_id": session_id, "status": "pending", "prompt_tokens": len(prompt_tokens),
                "quote": quote, "plan": plan}

    def _lease(self) -> Tuple[str, float]:
        return _uid(), _now() + ASSIGNMENT_LEASE_SECS

    def claim(self, device_id: str, max_decode_sessions: int = 64) -> dict:
        """Claim-time scheduling: in-flight prefill first, then a decode cohort of ready sessions
        whose decode group contains this device (one lease per session)."""
        self.reconcile_stale_leases()
        dev = self.db.one("SELECT * FROM devices WHERE device_id=?", (device_id,))
        if dev is None:
            raise NotFound(f"device {device_id} not registered")
        with self.db.tx() as c:
            row = c.execute("""SELECT a.*, j.prompt_tokens, j.max_tokens, j.temperature, j.top_p, j.model_id,
                               j.network_id, j.runtime_mode FROM inference_job_assignments a
                               JOIN inference_jobs j ON j.job_id=a.job_id
                               WHERE a.device_id=? AND a.phase='prefill' AND a.status='pending'
                               AND j.status IN ('pending','running') ORDER BY a.created_at LIMIT 1""",
                            (device_id,)).fetchone()
            if row is not None:
                row = dict(row)
                lease_id, exp = self._lease()
                c.execute("UPDATE inference_job_assignments SET status='leased', lease_id=?, lease_expires=?, "
                          "updated_at=? WHERE assignment_id=?", (lease_id, exp, _now(), row["assignment_id"]))
                c.execute("UPDATE inference_jobs SET status='running', updated_at=? WHERE job_id=?",
                          (_now(), row["job_id"]))
                c.execute("UPDATE inference_sessions SET status='prefilling', updated_at=? WHERE session_id=?",
                          (_now(), row["session_id"]))
                return {"kind": "prefill", "lease_id": lease_id, "lease_expires": exp,
                        "assignments": [self._assignment_view(row)]}
            ready = [dict(r) for r in c.execute(
                """SELECT q.*, j.prompt_tokens, j.max_tokens, j.temperature, j.top_p, j.model_id, j.runtime_mode,
                   g.member_device_ids FROM inference_decode_queue q JOIN inference_jobs j ON j.job_id=q.job_id
                   JOIN inference_serving_groups g ON g.session_id=q.session_id AND g.phase='decode'
                   WHERE q.status='ready' ORDER BY q.decode_steps_served, q.fairness_epoch LIMIT ?""",
                (max_decode_sessions * 4,)).fetchall()]
            cohort = [r for r in ready if device_id in loads(r["member_device_ids"], [])][:max_decode_sessions]
            if not cohort:
                return {"kind": "idle", "assignments": []}
            lease_id, exp = self._lease()
            out = []
            for r in cohort:
                c.execute("UPDATE inference_decode_queue SET status='leased', lease_id=?, lease_device_id=?, "
                          "lease_expires=?, updated_at=? WHERE session_id=?",
                          (lease_id, device_id, exp, _now(), r["session_id"]))
                c.execute("UPDATE inference_sessions SET status='decoding', phase='decode', updated_at=? "
                          "WHERE session_id=?", (_now(), r["session_id"]))
                ckpt = c.execute("SELECT payload FROM inference_session_checkpoints WHERE session_id=?",
                                 (r["session_id"],)).fetchone()
                out.append({"job_id": r["job_id"], "session_id": r["session_id"], "phase": "decode",
                            "prompt_tokens": loads(r["prompt_tokens"]), "max_tokens": r["max_tokens"],
                            "temperature": r["temperature"], "top_p": r["top_p"], "model_id": r["model_id"],
                            "runtime_mode": r["runtime_mode"], "has_checkpoint": ckpt is not None})
            c.execute("INSERT INTO inference_decode_batch_events (network_id, device_id, batch_size, kv_tokens, "
                      "created_at) VALUES (?,?,?,?,?)", (cohort[0]["network_id"], device_id, len(out),
                                                         sum(r["kv_seq_len"] for r in cohort), _now()))
            return {"kind": "decode", "lease_id": lease_id, "lease_expires": exp, "assignments": out}

    @staticmethod
    def _assignment_view(row: dict) -> dict:
        return {k: row[k] for k in ("assignment_id", "job_id", "session_id", "device_id", "phase", "segment_id",
                                    "group_id", "shard_column_start", "shard_column_end", "worker_position",
                                    "total_workers", "model_id", "max_tokens", "temperature", "top_p",
                                    "runtime_mode")} | {"prompt_tokens": loads(row["prompt_tokens"])}

    def acknowledge(self, job_id: str, device_id: str) -> dict:
        with self.db.tx() as c:
            c.execute("UPDATE inference_job_assignments SET status='acked', updated_at=? WHERE job_id=? AND "
                      "device_id=? AND status='leased'", (_now(), job_id, device_id))
        return {"job_id": job_id, "acknowledged": True}

    def renew_lease(self, lease_id: str) -> dict:
        exp = _now() + ASSIGNMENT_LEASE_SECS
        with self.db.tx() as c:
            n = c.execute("UPDATE inference_decode_queue SET lease_expires=? WHERE lease_id=?", (exp, lease_id)).rowcount
            n += c.execute("UPDATE inference_job_assignments SET lease_expires=? WHERE lease_id=?",
                           (exp, lease_id)).rowcount
        if n == 0:
            raise NotFound(f"lease {lease_id}")
        return {"lease_id": lease_id, "lease_expires": exp}

    def release_lease(self, lease_id: str, session_ids: Optional[List[str]] = None) -> dict:
        """Return leased decode sessions to the ready queue (e.g. after a worker error)."""
        with self.db.tx() as c:
            q = "UPDATE inference_decode_queue SET status='ready', lease_id=NULL, lease_device_id=NULL, " \
                "lease_expires=NULL, updated_at=? WHERE lease_id=? AND status IN ('leased','active')"
            args = [_now(), lease_id]
            if session_ids:
                q += " AND session_id IN (%s)" % ",".join("?" * len(session_ids))
                args += session_ids
            n = c.execute(q, args).rowcount
        return {"lease_id": lease_id, "released": n}

    def reconcile_stale_leases(self) -> int:
        now = _now()
        with self.db.tx() as c:
            n = c.execute("UPDATE inference_decode_queue SET status='ready', lease_id=NULL, lease_device_id=NULL, "
                          "lease_expires=NULL, updated_at=? WHERE status IN ('leased','active') AND lease_expires<?",
                          (now, now)).rowcount
            n += c.execute("UPDATE inference_job_assignments SET status='pending', lease_id=NULL, lease_expires=NULL "
                           "WHERE status IN ('leased','acked') AND lease_expires<?", (now,)).rowcount
        return n

    def report_progress(self, job_id: str, device_id: str, phase: str, completion_tokens: int,
                        kv_cache_seq_len: int = 0, time_to_first_token_ms: Optional[int] = None,
                        execution_time_ms: int = 0, kv_transfer: bool = False, **_) -> dict:
        job = self.db.one("SELECT * FROM inference_jobs WHERE job_id=?", (job_id,))
        if job is None:
            raise NotFound(f"job {job_id}")
        with self.db.tx() as c:
            if phase == "prefill":
                c.execute("UPDATE inference_job_assignments SET status='completed', execution_time_ms=?, updated_at=? "
                          "WHERE job_id=? AND device_id=? AND phase='prefill'",
                          (execution_time_ms, _now(), job_id, device_id))
                pending = c.execute("SELECT COUNT(*) FROM inference_job_assignments WHERE job_id=? AND phase='prefill' "
                                    "AND status!='completed'", (job_id,)).fetchone()[0]
                if pending == 0:
                    status = "blocked_on_transfer" if kv_transfer else "ready"
                    c.execute("UPDATE inference_decode_queue SET status=?, kv_seq_len=?, fairness_epoch="
                              "(SELECT COALESCE(MAX(fairness_epoch),0)+1 FROM inference_decode_queue), updated_at=? "
                              "WHERE job_id=?", (status, kv_cache_seq_len, _now(), job_id))
                    c.execute("UPDATE inference_sessions SET status='prefilled', kv_seq_len=?, updated_at=? "
                              "WHERE job_id=?", (kv_cache_seq_len, _now(), job_id))
                    c.execute("UPDATE inference_jobs SET ttft_ms=?, completion_tokens=?, updated_at=? WHERE job_id=?",
                              (time_to_first_token_ms, completion_tokens, _now(), job_id))
            else:
                c.execute("UPDATE inference_decode_queue SET status='active', decode_steps_served=?, kv_seq_len=?, "
                          "lease_expires=?, updated_at=? WHERE job_id=?",
                          (completion_tokens, kv_cache_seq_len, _now() + ASSIGNMENT_LEASE_SECS, _now(), job_id))
                c.execute("UPDATE inference_jobs SET completion_tokens=?, updated_at=? WHERE job_id=?",
                          (completion_tokens, _now(), job_id))
        return {"job_id": job_id, "accepted": True}

    def report_result(self, job_id: str, device_id: str, success: bool, generated_tokens: Optional[List[int]] = None,
                      error: Optional[str] = None, completion_tokens: int = 0, execution_time_ms: int = 0,
                      time_to_first_token_ms: Optional[int] = None, **_) -> dict:
        job = self.db.one("SELECT * FROM inference_jobs WHERE job_id=?", (job_id,))
        if job is None:
            raise NotFound(f"job {job_id}")
        if job["status"] in ("completed", "failed", "cancelled"):
            return {"job_id": job_id, "status": job["status"], "duplicate": True}
        cfg, total_bytes = self.model_config(job["model_id"])
        prompt = loads(job["prompt_tokens"])
        with self.db.tx() as c:
            if not success:
                self._fail_job(c, job, error or "worker reported failure")
                return {"job_id": job_id, "status": "failed"}
            c.execute("UPDATE inference_jobs SET status='completed', generated_tokens=?, completion_tokens=?, "
                      "execution_time_ms=?, ttft_ms=COALESCE(?, ttft_ms), updated_at=? WHERE job_id=?",
                      (dumps(generated_tokens or []), completion_tokens, execution_time_ms, time_to_first_token_ms,
                       _now(), job_id))
            c.execute("UPDATE inference_sessions SET status='completed', updated_at=? WHERE job_id=?", (_now(), job_id))
            c.execute("UPDATE inference_decode_queue SET status='completed', lease_id=NULL, updated_at=? WHERE job_id=?",
                      (_now(), job_id))
            members = [dict(r) for r in c.execute(
                "SELECT a.device_id, a.shard_column_start, a.shard_column_end, a.execution_time_ms, d.tier, "
                "d.contributed_memory FROM inference_job_assignments a LEFT JOIN devices d ON d.device_id=a.device_id "
                "WHERE a.job_id=? AND a.phase='prefill'", (job_id,)).fetchall()]
            credits = policy.credit_policy(
                len(prompt), completion_tokens, total_bytes, cfg.hidden_dim,
                [policy.AssignmentCreditInput(m["device_id"], max(m["execution_time_ms"] or execution_time_ms, 1),
                                              policy.TIER_CAPACITY_UNITS.get(m["tier"] or "tier2", 4),
                                              m["shard_column_start"], m["shard_column_end"],
                                              m["contributed_memory"] or 0) for m in members])
            settle = policy.consumption(len(prompt), completion_tokens, total_bytes)
            self._ledger(c, job["network_id"], job["submitter_device_id"], job_id, "credits_released",
                         job["credits_reserved"], {})
            self._ledger(c, job["network_id"], job["submitter_device_id"], job_id, "credits_spent",
                         settle["total_credits"], settle)
            for a in credits["assignments"]:
                self._ledger(c, job["network_id"], a["device_id"], job_id, "credits_earned", a["credits"], a)
            self._ledger(c, job["network_id"], job["submitter_device_id"], job_id, "job_completed", 0.0,
                         {"completion_tokens": completion_tokens})
        return {"job_id": job_id, "status": "completed", "settlement": settle}

    def _fail_job(self, c, job: dict, error: str) -> None:
        c.execute("UPDATE inference_jobs SET status='failed', error=?, updated_at=? WHERE job_id=?",
                  (error, _now(), job["job_id"]))
        c.execute("UPDATE inference_sessions SET status='failed', updated_at=? WHERE job_id=?", (_now(), job["job_id"]))
        c.execute("UPDATE inference_decode_queue SET status='failed', lease_id=NULL, updated_at=? WHERE job_id=?",
                  (_now(), job["job_id"]))
        self._ledger(c, job["network_id"], job["submitter_device_id"], job["job_id"], "credits_released",
                     job["credits_reserved"], {"reason": error})
        self._ledger(c, job["network_id"], job["submitter_device_id"], job["job_id"], "job_failed", 0.0,
                     {"error": error})

    def cancel_job(self, job_id: str) -> dict:
        job = self.db.one("SELECT * FROM inference_jobs WHERE job_id=?", (job_id,))
        if job is None:
            raise NotFound(f"job {job_id}")
        if job["status"] in ("completed", "failed", "cancelled"):
            return {"job_id": job_id, "status": job["status"]}
        with self.db.tx() as c:
            self._fail_job(c, job, "cancelled")
            c.execute("UPDATE inference_jobs SET status='cancelled' WHERE job_id=?", (job_id,))
        return {"job_id": job_id, "status": "cancelled"}

    def job_status(self, job_id: str) -> dict:
        job = self.db.one("SELECT * FROM inference_jobs WHERE job_id=?", (job_id,))
        if job is None:
            raise NotFound(f"job {job_id}")
        job["prompt_tokens"] = len(loads(job["prompt_tokens"]))
        job["generated_tokens"] = loads(job["generated_tokens"])
        job["plan"] = loads(job["plan"], {})
        q = self.db.one("SELECT * FROM inference_decode_queue WHERE job_id=?", (job_id,))
        job["decode_queue"] = q
        return job

    def observe_decode_queue(self, network_id: Optional[str] = None) -> dict:
        rows = self.db.query("SELECT * FROM inference_decode_queue" + (" WHERE network_id=?" if network_id else "") +
                             " ORDER BY decode_steps_served, fairness_epoch", [network_id] if network_id else [])
        counts = {s: 0 for s in DECODE_QUEUE_STATUSES}
        for r in rows:
            counts[r["status"]] = counts.get(r["status"], 0) + 1
        return {"entries": rows, "counts": counts}

    # ------------------------------------------------------------------------------------ checkpoints, KV
    def upload_session_checkpoint(self, job_id: str, session_id: str, payload: bytes, token_index: int = 0) -> dict:
        with self.db.tx() as c:
            c.execute("INSERT INTO inference_session_checkpoints VALUES (?,?,?,?,?) ON CONFLICT(job_id, session_id) "
                      "DO UPDATE SET payload=excluded.payload, token_index=excluded.token_index, "
                      "created_at=excluded.created_at", (job_id, session_id, payload, token_index, _now()))
        return {"job_id": job_id, "session_id": session_id, "bytes": len(payload),
                "sha256": hashlib.sha256(payload).hexdigest()}

    def download_session_checkpoint(self, job_id: str, session_id: str) -> bytes:
        r = self.db.one("SELECT payload FROM inference_session_checkpoints WHERE job_id=? AND session_id=?",
                        (job_id, session_id))
        if r is None:
            raise NotFound("no checkpoint for session")
        return r["payload"]

    def report_kv_transfer(self, job_id: str, session_id: str, source_device_id: str, target_device_id: str,
                           status: str = "pending", transfer_id: Optional[str] = None) -> dict:
        tid = transfer_id or _uid()
        with self.db.tx() as c:
            c.execute("INSERT INTO inference_session_kv_transfers VALUES (?,?,?,?,?,?,?,?) ON CONFLICT(transfer_id) "
                      "DO UPDATE SET status=excluded.status, updated_at=excluded.updated_at",
                      (tid, job_id, session_id, source_device_id, target_device_id, status, _now(), _now()))
            if status == "completed":
                c.execute("UPDATE inference_decode_queue SET status='ready', updated_at=? WHERE session_id=? AND "
                          "status='blocked_on_transfer'", (_now(), session_id))
                c.execute("INSERT INTO inference_session_kv_residency VALUES (?,?,NULL,?) ON CONFLICT(session_id, "
                          "device_id) DO UPDATE SET updated_at=excluded.updated_at",
                          (session_id, target_device_id, _now()))
        return {"transfer_id": tid, "status": status}

    def pending_kv_transfers(self, device_id: str) -> List[dict]:
        return self.db.query("SELECT * FROM inference_session_kv_transfers WHERE target_device_id=? AND "
                             "status='pending' ORDER BY created_at", (device_id,))

    def upload_kv_payload(self, transfer_id: str, payload: bytes) -> dict:
        with self.db.tx() as c:
            c.execute("INSERT INTO inference_session_kv_transfer_payloads VALUES (?,?,?) ON CONFLICT(transfer_id) DO "
                      "UPDATE SET payload=excluded.payload", (transfer_id, payload, _now()))
        return {"transfer_id": transfer_id, "bytes": len(payload)}

    def download_kv_payload(self, transfer_id: str) -> bytes:
        r = self.db.one("SELECT payload FROM inference_session_kv_transfer_payloads WHERE transfer_id=?", (transfer_id,))
        if r is None:
            raise NotFound(f"no payload for transfer {transfer_id}")
        return r["payload"]

    # ------------------------------------------------------------------------------------ failover / presence
    def evaluate_failover(self, lost_device_ids: List[str]) -> List[dict]:
        """Regroup every job touched by the lost devices; returns the decisions taken."""
        lost = set(lost_device_ids)
        decisions = []
        jobs = self.db.query("SELECT * FROM inference_jobs WHERE status IN ('pending','running')")
        for job in jobs:
            plan = loads(job["plan"], {})
            groups = {g["phase"]: g for g in plan.get("execution_groups", [])}
            parts = {m["device_id"] for g in groups.values() for m in g["members"]}
            if not parts & lost:
                continue
            q = self.db.one("SELECT * FROM inference_decode_queue WHERE job_id=?", (job["job_id"],))
            phase = "prefill" if q is None or q["status"] == "blocked_on_prefill" else "decode"
            with self.db.tx() as c:
                if phase == "prefill":
                    self._fail_job(c, job, f"prefill group lost devices {sorted(parts & lost)}")
                    d = {"job_id": job["job_id"], "strategy": "fail", "recovery_state": "failed",
                         "resume_mode": "none", "lost_device_ids": sorted(parts & lost)}
                else:
                    d = self._decode_failover(c, job, plan, groups["decode"], lost, q)
                c.execute("INSERT INTO inference_regroup_events (job_id, session_id, decision, details, created_at) "
                          "VALUES (?,?,?,?,?)", (job["job_id"], q["session_id"] if q else None, d["strategy"],
                                                 dumps(d), _now()))
            decisions.append(d)
        return decisions

    def _decode_failover(self, c, job, plan, group, lost, q) -> dict:
        members = group["members"]
        survivors = [m for m in members if m["device_id"] not in lost]
        lost_ids = sorted(m["device_id"] for m in members if m["device_id"] in lost)
        has_ckpt = c.execute("SELECT 1 FROM inference_session_checkpoints WHERE session_id=?",
                             (q["session_id"],)).fetchone() is not None
        resume = "requires_checkpoint_transfer" if has_ckpt else "none"
        # replacement candidates: online ring members of the network not already serving this group
        ring = [dict(r) for r in c.execute(
            "SELECT m.device_id, m.column_start, m.column_end FROM ring_members m JOIN devices d ON "
            "d.device_id=m.device_id WHERE m.network_id=? AND d.status='online'", (job["network_id"],)).fetchall()]
        in_group = {m["device_id"] for m in members}
        spare = [r for r in ring if r["device_id"] not in in_group and r["device_id"] not in lost]
        strategy, new_members = "fail", None
        if spare and len(spare) >= len(lost_ids) and has_ckpt:
            repl = spare[:len(lost_ids)]
            new_members = survivors + [{**m, "device_id": r["device_id"]} for m, r in
                                       zip([m for m in members if m["device_id"] in lost], repl)]
            strategy = "replace"
        elif survivors and has_ckpt:
            covered = sorted((m["shard_column_start"], m["shard_column_end"]) for m in survivors)
            full = covered and covered[0][0] == 0 and all(covered[i][1] == covered[i + 1][0]
                                                          for i in range(len(covered) - 1))
            cfg, _ = self.model_config(job["model_id"])
            if full and covered[-1][1] == cfg.hidden_dim:
                new_members = survivors
                strategy = "shrink"
            elif len(survivors) >= 1:
                # survivors re-shard the full model (FullReplica-capable workers)
                new_members = [{**m, "shard_column_start": 0, "shard_column_end": cfg.hidden_dim,
                                "worker_position": i, "total_workers": 1} for i, m in enumerate(survivors[:1])]
                strategy = "shrink"
        if strategy == "fail":
            self._fail_job(c, job, f"decode group lost devices {lost_ids} without a recoverable regroup")
            return {"job_id": job["job_id"], "strategy": "fail", "recovery_state": "failed", "resume_mode": "none",
                    "lost_device_ids": lost_ids}
        group = dict(group)
        group["members"] = new_members
        plan = dict(plan)
        plan["execution_groups"] = [g if g["phase"] != "decode" else group for g in plan["execution_groups"]]
        c.execute("UPDATE inference_jobs SET plan=?, updated_at=? WHERE job_id=?", (dumps(plan), _now(), job["job_id"]))
        c.execute("UPDATE inference_serving_groups SET member_device_ids=? WHERE group_id=?",
                  (dumps([m["device_id"] for m in new_members]), group["group_id"]))
        c.execute("UPDATE inference_decode_queue SET status='ready', lease_id=NULL, lease_device_id=NULL, "
                  "lease_expires=NULL, updated_at=? WHERE session_id=?", (_now(), q["session_id"]))
        return {"job_id": job["job_id"], "strategy": strategy, "recovery_state": "resume_ready",
                "resume_mode": resume, "lost_device_ids": lost_ids,
                "participant_device_ids": [m["device_id"] for m in new_members]}

    def presence_sweep(self, now: Optional[float] = None) -> List[str]:
        """Mark devices silent for longer than the stale timeout as stale and regroup their work."""
        now = _now() if now is None else now
        stale = [r["device_id"] for r in self.db.query(
            "SELECT device_id FROM devices WHERE status='online' AND last_heartbeat < ?", (now - self.stale_timeout_s,))]
        if stale:
            with self.db.tx() as c:
                c.executemany("UPDATE devices SET status='stale' WHERE device_id=?", [(d,) for d in stale])
            self.evaluate_failover(stale)
        return stale

    # ------------------------------------------------------------------------------------ status
    def network_scheduler_status(self, network_id: str) -> dict:
        q = self.observe_decode_queue(network_id)
        jobs = self.db.query("SELECT status, COUNT(*) AS n FROM inference_jobs WHERE network_id=? GROUP BY status",
                             (network_id,))
        peak = self.db.one("SELECT MAX(batch_size) AS p FROM inference_decode_batch_events WHERE network_id=?",
                           (network_id,))
        topo = self.db.query("SELECT DISTINCT model_id FROM ring_members WHERE network_id=?", (network_id,))
        blockers = []
        for t in topo:
            if not self.topology(network_id, t["model_id"])["stable"]:
                blockers.append(f"ring for {t['model_id']} is not stable")
        return {"network_id": network_id, "jobs": {j["status"]: j["n"] for j in jobs},
                "decode_queue": q["counts"], "peak_batch_size": (peak or {}).get("p") or 0,
                "readiness_blockers": blockers,
                "regroup_events": self.db.query("SELECT * FROM inference_regroup_events ORDER BY id DESC LIMIT 20")}

    def job_scheduler_status(self, job_id: str) -> dict:
        st = self.job_status(job_id)
        ev = self.db.query("SELECT * FROM inference_scheduler_events WHERE job_id=? ORDER BY id", (job_id,))
        rg = self.db.query("SELECT * FROM inference_regroup_events WHERE job_id=? ORDER BY id", (job_id,))
        return {"job": st, "scheduler_events": ev, "regroup_events": rg}
