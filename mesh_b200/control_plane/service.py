"""Control-plane services (business logic behind the HTTP API).

Behaviour restated from the reference control plane (``control-plane/src``):

* device registration and heartbeat (``services/device_service.rs``, ``api/routes.rs``);
* ring topology: sequential positions, weighted GQA-aligned column ranges, neighbours, version
  counter, handoffs and callbacks (``services/ring_manager.rs:140-1091``,
  ``services/topology_notifier.rs``);
* execution planning: prefill and decode members chosen separately under the model's execution
  layout rules and scored per runtime mode (``planner.py``, ``services/planner.rs:49-372``); a
  decode group that differs from the prefill group receives the KV by checkpoint handoff;
* submit: tokenize, quote + reserve credits, persist job / session / groups / assignments and a
  decode queue entry ``blocked_on_prefill`` in one transaction (``api/inference.rs:383-765``);
* claim: the claim-time scheduler (``scheduler.py``) orders this worker's prefill assignments and
  decode-queue entries (in-flight prefill groups first, blocked reasons, soft caps), then a
  decode claim leases the cohort of runnable sessions, 60 s leases (``api/inference.rs:4567-4925``,
  ``services/scheduler.rs:119-197``); renew / release leases;
* progress: PrefillComplete moves the queue entry to ``ready`` (co-located) or
  ``blocked_on_transfer`` (handoff) (``api/inference.rs:5782-6412``);
* result: completion, settlement through the credit policy, ledger events (``:5320-5781``);
* failover: the failover engine (``failover.py``): prefill loss -> fail and release credits;
  decode loss -> the decode group re-planned on the live ring, else the survivors that still cover
  the columns; resume immediately, after a live KV handoff or after a checkpoint transfer
  (``services/failover.rs:174-700``); terminal sessions and orphaned leases are cleaned up
  (``:2158-2312``);
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
from . import failover as fo
from . import planner as planner_mod
from . import policy
from . import scheduler as sched
from .db import Database, dumps, loads
from .layout import LayoutError, Member, ModelManifest
from .provider import contract_for_device

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
    def __init__(self, db: Optional[Database] = None, model_store: Optional[str] = None, key_path: Optional[str] = None):
        from .certificate import ControlPlaneKeypair
        self.db = db or Database()
        self.model_store = model_store
        # signs device certificates at registration; MESH_CONTROL_PLANE_KEY names a key file to keep
        key_path = key_path or os.environ.get("MESH_CONTROL_PLANE_KEY")
        self.keypair = ControlPlaneKeypair.load_or_generate(key_path) if key_path else ControlPlaneKeypair.generate()
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

    def manifest(self, model_id: str) -> ModelManifest:
        """The planning view of a model: ``model.json`` (with its ``execution_layout`` rules) from
        the model store, else the attention geometry of the built-in preset."""
        if self.model_store:
            p = os.path.join(self.model_store, model_id, "model.json")
            if os.path.exists(p):
                m = json.load(open(p))
                m.setdefault("model_id", model_id)
                m.setdefault("total_model_bytes", self.model_config(model_id)[1])
                try:
                    return ModelManifest.from_json(m)
                except LayoutError as e:
                    raise ApiError(str(e)) from e
        cfg, total = self.model_config(model_id)
        return ModelManifest(model_id, cfg.hidden_dim, cfg.num_heads, cfg.num_kv_heads, total, cfg.num_layers)

    def _members(self, network_id: str, model_id: str, exclude=()) -> List[Member]:
        """Online ring members of a model as planner members (contract from the device's
        advertised capabilities, capacity units from its tier)."""
        rows = self.db.query(
            "SELECT m.device_id, m.position, m.column_start, m.column_end, m.contributed_memory, d.tier, d.provider, "
            "d.capabilities, d.status, d.tensor_plane_addr FROM ring_members m JOIN devices d ON d.device_id=m.device_id "
            "WHERE m.network_id=? AND m.model_id=? AND m.status='active' ORDER BY m.position", (network_id, model_id))
        out = []
        for r in rows:
            if r["device_id"] in exclude or r["status"] != "online" or r["column_end"] <= r["column_start"]:
                continue
            out.append(Member(r["device_id"], r["position"], r["column_start"], r["column_end"],
                              contributed_memory=r["contributed_memory"] or 0,
                              assigned_capacity_units=policy.TIER_CAPACITY_UNITS.get(r["tier"] or "tier2", 4),
                              backend_contract=contract_for_device(r["provider"] or "cpu", loads(r["capabilities"], {})),
                              listen_addrs=["dataplane://" + (r["tensor_plane_addr"] or r["device_id"])]))
        return out

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
        """Register (or re-register) a device. With its ed25519 public key (64 hex characters) the
        control plane issues a signed 30-day certificate (``certificate.py``) and returns it with
        its own public key; a device-supplied ``certificate`` is ignored."""
        if not device_id:
            raise ApiError("device_id cannot be empty")
        if network_id is not None:
            if not network_id:
                raise ApiError("network_id cannot be empty")
            if not self.db.query("SELECT 1 FROM networks WHERE network_id=?", (network_id,)):
                raise NotFound(f"network {network_id} not found")
        cert_hex = ""
        if public_key:
            try:
                pk = bytes.fromhex(public_key)
            except ValueError:
                raise ApiError("public_key must be hex")
            if len(pk) != 32:
                raise ApiError("public_key must be 32 bytes (Ed25519)")
            cert_hex = self.keypair.generate_certificate(device_id, network_id or "", pk).hex()
        certificate = cert_hex
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
            c.execute("UPDATE devices SET public_key=?, certificate=? WHERE device_id=?",
                      (public_key, certificate, device_id))
        return {"device_id": device_id, "status": "online", "certificate": certificate,
                "control_plane_public_key": self.keypair.public_key().hex()}

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
        """Prefill and decode groups for a new session (``planner.plan``); Conflict when the live
        ring cannot form a legal group."""
        topo = self.topology(network_id, model_id)
        if not topo["stable"]:
            raise Conflict("ring is not stable: no full column coverage by online workers")
        try:
            p = planner_mod.plan(self.manifest(model_id), self._members(network_id, model_id))
        except (planner_mod.PlanningError, LayoutError) as e:
            raise Conflict(str(e)) from e
        out = p.to_json(model_id, session_id)
        out["topology_version"] = topo["version"]
        return out

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
            for i, m in enumerate(plan["execution_groups"][0]["members"]):
                c.execute("""INSERT INTO inference_job_assignments (assignment_id, job_id, session_id, device_id, phase,
                             segment_id, group_id, status, shard_column_start, shard_column_end, worker_position,
                             total_workers, created_at, updated_at) VALUES (?,?,?,?,'prefill',?,?,'pending',?,?,?,?,?,?)""",
                          (_uid(), job_id, session_id, m["device_id"], plan["segments"][0]["segment_id"],
                           plan["execution_groups"][0]["group_id"], m["shard_column_start"], m["shard_column_end"],
                           i, m["total_workers"], now, now))
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

    @staticmethod
    def _iso(t: Optional[float]) -> str:
        import datetime as _dt
        return _dt.datetime.fromtimestamp(t or 0.0, _dt.timezone.utc).strftime("%Y-%m-%dT%H:%M:%S.%fZ")

    def _claim_candidates(self, c, device_id: str) -> Tuple[List[sched.Candidate], dict, sched.Snapshot]:
        """The scheduler's view of what ``device_id`` could take: its pending prefill assignments
        and the decode-queue entries whose decode group contains it, with group and cohort state."""
        iso = self._iso
        cands: List[sched.Candidate] = []
        rows = {}
        inflight_by_model: Dict[str, set] = {}
        for r in c.execute("SELECT a.job_id, j.model_id FROM inference_job_assignments a JOIN inference_jobs j ON "
                           "j.job_id=a.job_id WHERE a.phase='prefill' AND a.status IN ('leased','acked') AND "
                           "j.status IN ('pending','running')").fetchall():
            inflight_by_model.setdefault(r["model_id"], set()).add(r["job_id"])
        for r in c.execute("""SELECT a.*, j.prompt_tokens, j.max_tokens, j.temperature, j.top_p, j.model_id, j.network_id,
                              j.runtime_mode, j.submitter_device_id, j.created_at AS job_created FROM
                              inference_job_assignments a JOIN inference_jobs j ON j.job_id=a.job_id WHERE a.device_id=?
                              AND a.phase='prefill' AND a.status='pending' AND j.status IN ('pending','running')""",
                           (device_id,)).fetchall():
            r = dict(r)
            st = [x["status"] for x in c.execute("SELECT status FROM inference_job_assignments WHERE job_id=? AND "
                                                 "phase='prefill'", (r["job_id"],)).fetchall()]
            others = inflight_by_model.get(r["model_id"], set()) - {r["job_id"]}
            cands.append(sched.Candidate(
                assignment_id=r["assignment_id"], job_id=r["job_id"], session_id=r["session_id"], phase="prefill",
                group_status="prefill_member", model_id=r["model_id"], ring_position=r["worker_position"] or 0,
                runtime_mode=r["runtime_mode"] or "throughput_first", submitted_by_device_id=r["submitter_device_id"] or "",
                created_at=iso(r["job_created"]), assigned_at=iso(r["created_at"]),
                prefill_group_total_members=len(st),
                prefill_group_leased_members=sum(1 for x in st if x in ("leased", "acked")),
                prefill_group_active_members=sum(1 for x in st if x == "completed"),
                model_prefill_inflight_groups=len(others)))
            rows[r["assignment_id"]] = ("prefill", r)
        q = [dict(r) for r in c.execute(
            """SELECT q.*, j.prompt_tokens, j.max_tokens, j.temperature, j.top_p, j.model_id, j.runtime_mode,
               j.submitter_device_id, j.created_at AS job_created, g.member_device_ids FROM inference_decode_queue q
               JOIN inference_jobs j ON j.job_id=q.job_id JOIN inference_serving_groups g ON g.session_id=q.session_id
               AND g.phase='decode' WHERE q.status IN ('ready','leased','active','blocked_on_transfer',
               'blocked_on_prefill') AND j.status IN ('pending','running')""").fetchall()]
        cohorts: Dict[tuple, dict] = {}
        for r in q:
            key = tuple(sorted(loads(r["member_device_ids"], [])))
            st = cohorts.setdefault(key, dict(ready=0, blocked=0, blocked_prefill=0, leased=0, active=0, oldest=None))
            if r["status"] == "ready":
                st["ready"] += 1
                t = iso(r["updated_at"])
                st["oldest"] = t if st["oldest"] is None else min(st["oldest"], t)
            elif r["status"] == "blocked_on_transfer":
                st["blocked"] += 1
            elif r["status"] == "blocked_on_prefill":
                st["blocked_prefill"] += 1
                st["blocked"] += 1
            elif r["status"] == "leased":
                st["leased"] += 1
            elif r["status"] == "active":
                st["active"] += 1
        for r in q:
            key = tuple(sorted(loads(r["member_device_ids"], [])))
            if device_id not in key or r["status"] == "blocked_on_prefill":
                continue
            st = cohorts[key]
            own = r["lease_device_id"] == device_id
            if r["status"] == "ready":
                gs = "decode_ready"
            elif own:
                gs = "decode_active"
            else:
                gs = "decode_member"
            cands.append(sched.Candidate(
                assignment_id="decode:" + r["session_id"], job_id=r["job_id"], session_id=r["session_id"],
                phase="decode", group_status=gs, model_id=r["model_id"],
                runtime_mode=r["runtime_mode"] or "throughput_first", submitted_by_device_id=r["submitter_device_id"] or "",
                created_at=iso(r["job_created"]), decode_queue_status=r["status"], decode_ready_at=iso(r["updated_at"]),
                decode_lease_owner_device_id=r["lease_device_id"], decode_lease_expires_at=(
                    iso(r["lease_expires"]) if r["lease_expires"] else None),
                decode_updated_at=iso(r["updated_at"]), decode_cohort_ready_sessions=st["ready"],
                decode_cohort_blocked_sessions=st["blocked"], decode_cohort_blocked_prefill_sessions=st["blocked_prefill"],
                decode_cohort_oldest_ready_at=st["oldest"], decode_cohort_leased_sessions=st["leased"],
                decode_cohort_active_sessions=st["active"]))
            rows["decode:" + r["session_id"]] = ("decode", r, key)
        snap = sched.Snapshot()
        for r in c.execute("SELECT submitter_device_id, model_id, COUNT(*) AS n FROM inference_jobs WHERE status="
                           "'running' GROUP BY submitter_device_id, model_id").fetchall():
            snap.active_jobs_by_submitter[r["submitter_device_id"] or ""] = \
                snap.active_jobs_by_submitter.get(r["submitter_device_id"] or "", 0) + r["n"]
            snap.active_jobs_by_model[r["model_id"]] = snap.active_jobs_by_model.get(r["model_id"], 0) + r["n"]
        online = c.execute("SELECT COUNT(*), COALESCE(SUM(CASE tier WHEN 'tier0' THEN 1 WHEN 'tier1' THEN 2 "
                           "WHEN 'tier3' THEN 8 WHEN 'tier4' THEN 16 ELSE 4 END), 0) FROM devices WHERE "
                           "status='online'").fetchone()
        snap.online_worker_count = max(1, online[0])
        snap.online_capacity_units = max(1, online[1])
        return cands, rows, snap

    def claim(self, device_id: str, max_decode_sessions: int = 64, mode: str = "fit_first") -> dict:
        """Claim-time scheduling (``scheduler.select_claim``): an in-flight prefill group first, then a
        prefill whose decode cohort waits, then the best-ranked runnable work; a decode claim
        leases the cohort of runnable sessions sharing the chosen session's decode group (one lease)."""
        self.reconcile_stale_leases()
        dev = self.db.one("SELECT * FROM devices WHERE device_id=?", (device_id,))
        if dev is None:
            raise NotFound(f"device {device_id} not registered")
        with self.db.tx() as c:
            cands, rows, snap = self._claim_candidates(c, device_id)
            decision = sched.select_claim(cands, device_id, self._iso(_now()), mode, snap=snap)
            if decision.blocked:
                reasons: Dict[str, int] = {}
                for b in decision.blocked:
                    reasons[b.reason] = reasons.get(b.reason, 0) + 1
                c.execute("INSERT INTO inference_scheduler_events (network_id, job_id, event, details, created_at) "
                          "VALUES (?,?,?,?,?)", (dev["network_id"], None, "claim_blocked",
                                                 dumps({"device_id": device_id, "reasons": reasons}), _now()))
            sel = decision.selected_assignment_id
            if sel is None:
                return {"kind": "idle", "assignments": [],
                        "blocked": [{"session_id": b.session_id, "reason": b.reason} for b in decision.blocked]}
            if rows[sel][0] == "prefill":
                row = rows[sel][1]
                lease_id, exp = self._lease()
                c.execute("UPDATE inference_job_assignments SET status='leased', lease_id=?, lease_expires=?, "
                          "updated_at=? WHERE assignment_id=?", (lease_id, exp, _now(), row["assignment_id"]))
                c.execute("UPDATE inference_jobs SET status='running', updated_at=? WHERE job_id=?",
                          (_now(), row["job_id"]))
                c.execute("UPDATE inference_sessions SET status='prefilling', updated_at=? WHERE session_id=?",
                          (_now(), row["session_id"]))
                return {"kind": "prefill", "lease_id": lease_id, "lease_expires": exp,
                        "assignments": [self._assignment_view(row)]}
            key = rows[sel][2]
            now_iso = self._iso(_now())
            cohort = [cd for cd in cands if cd.phase == "decode" and rows[cd.assignment_id][2] == key and
                      not isinstance(sched.classify(cd, device_id, now_iso), tuple)]
            cohort.sort(key=lambda cd: (sched.decode_session_order_time(sched.Runnable(cd, cd.decode_ready_at or "")),
                                        cd.assignment_id))
            cohort = cohort[:max_decode_sessions]
            lease_id, exp = self._lease()
            out = []
            for cd in cohort:
                r = rows[cd.assignment_id][1]
                attached = cd.decode_queue_status in ("leased", "active")
                if not attached:
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
                            "runtime_mode": r["runtime_mode"], "has_checkpoint": ckpt is not None,
                            "attached_to_lease": r["lease_id"] if attached else None})
            c.execute("INSERT INTO inference_decode_batch_events (network_id, device_id, batch_size, kv_tokens, "
                      "created_at) VALUES (?,?,?,?,?)", (rows[cohort[0].assignment_id][1]["network_id"], device_id,
                                                         len(out), sum(rows[cd.assignment_id][1]["kv_seq_len"]
                                                                       for cd in cohort), _now()))
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
                    handoff = loads(job["plan"], {}).get("kv_transfer_policy") == "checkpoint_handoff"
                    has_ckpt = c.execute("SELECT 1 FROM inference_session_checkpoints WHERE job_id=?",
                                         (job_id,)).fetchone() is not None
                    status = "blocked_on_transfer" if (kv_transfer or (handoff and not has_ckpt)) else "ready"
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
    def upload_session_checkpoint(self, job_id: str, session_id: str, payload: bytes, token_index: int = 0,
                                  source_device_id: Optional[str] = None) -> dict:
        with self.db.tx() as c:
            c.execute("INSERT INTO inference_session_checkpoints VALUES (?,?,?,?,?,?) ON CONFLICT(job_id, session_id) "
                      "DO UPDATE SET payload=excluded.payload, token_index=excluded.token_index, "
                      "created_at=excluded.created_at, source_device_id=excluded.source_device_id",
                      (job_id, session_id, payload, token_index, _now(), source_device_id))
            # a checkpoint-handoff decode group waiting for the prefill's KV can start now
            c.execute("UPDATE inference_decode_queue SET status='ready', updated_at=? WHERE session_id=? AND "
                      "status='blocked_on_transfer' AND NOT EXISTS (SELECT 1 FROM inference_session_kv_transfers t "
                      "WHERE t.session_id=? AND t.status='pending')", (_now(), session_id, session_id))
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
        """Regroup every running job touched by the lost devices (``failover.FailoverEngine``);
        returns the decisions taken."""
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
                d = self._failover_decision(c, job, plan, groups, phase, lost, q)
                c.execute("INSERT INTO inference_regroup_events (job_id, session_id, decision, details, created_at) "
                          "VALUES (?,?,?,?,?)", (job["job_id"], q["session_id"] if q else None, d["strategy"],
                                                 dumps(d), _now()))
            decisions.append(d)
        return decisions

    @staticmethod
    def _plan_members(group: dict) -> List[Member]:
        return [Member(m["device_id"], m.get("worker_position", i), m["shard_column_start"], m["shard_column_end"],
                       contributed_memory=m.get("contributed_memory", 0),
                       assigned_capacity_units=m.get("assigned_capacity_units", 4),
                       listen_addrs=["dataplane://" + m["device_id"]])
                for i, m in enumerate(group["members"])]

    def _failover_decision(self, c, job, plan, groups, phase, lost, q) -> dict:
        group = groups["prefill" if phase == "prefill" else "decode"]
        members = self._plan_members(group)
        sess = self.db.one("SELECT * FROM inference_sessions WHERE job_id=?", (job["job_id"],)) or {}
        ck = c.execute("SELECT source_device_id, created_at FROM inference_session_checkpoints WHERE job_id=? "
                       "ORDER BY created_at DESC LIMIT 1", (job["job_id"],)).fetchone()
        ck_dev = None
        if ck is not None:
            src = ck["source_device_id"] or sess.get("kv_owner_device_id")
            st = c.execute("SELECT status FROM devices WHERE device_id=?", (src,)).fetchone()
            # the control plane stores the checkpoint payload itself, so it survives its source device
            ck_dev = src if (st is not None and st["status"] == "online" and src not in lost) else "control-plane"
        session = fo.SessionView(
            session_id=sess.get("session_id", ""), status="decode_active" if (q and q["status"] in ("leased", "active"))
            else "decode_ready", phase=phase, participants=[m.device_id for m in members],
            kv_owner_device_id=sess.get("kv_owner_device_id") or members[0].device_id,
            kv_sequence_position=int(sess.get("kv_seq_len") or 0), latest_checkpoint_device_id=ck_dev,
            latest_checkpoint_created_at=self._iso(ck["created_at"]) if ck is not None else None,
            segment_id=f"segment-{sess.get('session_id', '')}-{phase}")
        refreshed = None
        if phase == "decode":
            live = self._members(job["network_id"], job["model_id"], exclude=lost)
            try:
                cur = planner_mod.Plan(plan.get("plan_id", ""), plan.get("runtime_mode", "latency_first"), [],
                                       [m for m in members if m.device_id not in lost] or members, "", "")
                re = planner_mod.refresh_decode_plan(self.manifest(job["model_id"]), cur, live)
                if all(m.device_id not in lost for m in re.decode):
                    refreshed = ([m.device_id for m in re.decode], planner_mod.select_kv_owner(re.decode))
                    known = {m.device_id for m in members}
                    members = members + [m for m in re.decode if m.device_id not in known]
            except (planner_mod.PlanningError, LayoutError):
                refreshed = None
        transfers = [fo.KvTransfer(f"segment-{t['session_id']}-decode", t["source_device_id"], t["target_device_id"],
                                   "live_kv_handoff", t["status"], int(sess.get("kv_seq_len") or 0))
                     for t in c.execute("SELECT * FROM inference_session_kv_transfers WHERE job_id=?",
                                        (job["job_id"],)).fetchall()]
        support = fo.SupportGroups(kv={m.device_id for m in members}, recovery={m.device_id for m in members})
        d = fo.FailoverEngine().evaluate(session, members, sorted(lost), q["status"] if q else None, transfers,
                                         refreshed, support if plan.get("live_kv_handoff") else None)
        out = d.to_json()
        out["job_id"] = job["job_id"]
        out["participant_device_ids"] = d.target_participant_device_ids
        if d.recovery_state == "failed":
            self._fail_job(c, job, d.reason)
            return out
        if d.recovery_state == "healthy":
            return out
        by_id = {m.device_id: m for m in members}
        new_members = []
        for i, dev_id in enumerate(d.target_participant_device_ids):
            m = by_id[dev_id]
            new_members.append({**m.to_json(), "worker_position": i,
                                "total_workers": len(d.target_participant_device_ids)})
        group = dict(group)
        group["members"] = new_members
        plan = dict(plan)
        plan["execution_groups"] = [g if g["phase"] != "decode" else group for g in plan["execution_groups"]]
        c.execute("UPDATE inference_jobs SET plan=?, updated_at=? WHERE job_id=?", (dumps(plan), _now(), job["job_id"]))
        c.execute("UPDATE inference_serving_groups SET member_device_ids=? WHERE group_id=?",
                  (dumps(d.target_participant_device_ids), group["group_id"]))
        c.execute("UPDATE inference_sessions SET kv_owner_device_id=?, updated_at=? WHERE job_id=?",
                  (d.next_kv_owner_device_id, _now(), job["job_id"]))
        c.execute("UPDATE inference_decode_queue SET status=?, lease_id=NULL, lease_device_id=NULL, lease_expires=NULL, "
                  "updated_at=? WHERE session_id=?", (d.decode_queue_status, _now(), q["session_id"]))
        if d.resume_mode in ("requires_live_kv_transfer", "requires_checkpoint_transfer"):
            for dev_id in d.replacement_device_ids or d.target_participant_device_ids:
                c.execute("INSERT INTO inference_session_kv_transfers VALUES (?,?,?,?,?,'pending',?,?)",
                          (_uid(), job["job_id"], q["session_id"], d.transfer_source_device_id, dev_id, _now(), _now()))
        return out

    def cleanup_terminal_state(self) -> dict:
        """Release what finished or failed sessions still hold: decode-queue leases of terminal jobs,
        assignments leased to devices that are gone, pending KV transfers of terminal jobs
        (``failover.rs:2158-2312``)."""
        now = _now()
        with self.db.tx() as c:
            q = c.execute("UPDATE inference_decode_queue SET lease_id=NULL, lease_device_id=NULL, lease_expires=NULL, "
                          "status=CASE WHEN status IN ('completed','failed') THEN status ELSE 'failed' END, updated_at=? "
                          "WHERE job_id IN (SELECT job_id FROM inference_jobs WHERE status IN "
                          "('completed','failed','cancelled')) AND (lease_id IS NOT NULL OR status NOT IN "
                          "('completed','failed'))", (now,)).rowcount
            a = c.execute("UPDATE inference_job_assignments SET status='pending', lease_id=NULL, lease_expires=NULL, "
                          "updated_at=? WHERE status IN ('leased','acked') AND device_id NOT IN (SELECT device_id FROM "
                          "devices WHERE status='online')", (now,)).rowcount
            t = c.execute("UPDATE inference_session_kv_transfers SET status='cancelled', updated_at=? WHERE "
                          "status='pending' AND job_id IN (SELECT job_id FROM inference_jobs WHERE status IN "
                          "('completed','failed','cancelled'))", (now,)).rowcount
        return {"queue_leases_released": q, "orphaned_assignments": a, "transfers_cancelled": t}

    def presence_sweep(self, now: Optional[float] = None) -> List[str]:
        """Mark devices silent for longer than the stale timeout as stale and regroup their work."""
        now = _now() if now is None else now
        stale = [r["device_id"] for r in self.db.query(
            "SELECT device_id FROM devices WHERE status='online' AND last_heartbeat < ?", (now - self.stale_timeout_s,))]
        if stale:
            with self.db.tx() as c:
                c.executemany("UPDATE devices SET status='stale' WHERE device_id=?", [(d,) for d in stale])
            self.evaluate_failover(stale)
            self.cleanup_terminal_state()
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
