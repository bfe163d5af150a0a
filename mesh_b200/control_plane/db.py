"""SQLite persistence of the control plane.

Table names follow the reference's migrations (``control-plane/migrations``): devices, networks,
ledger_events, inference_jobs, inference_job_assignments, inference_sessions,
inference_serving_groups, inference_decode_queue, inference_decode_batch_events,
inference_scheduler_events, inference_regroup_events, inference_session_checkpoints,
inference_session_kv_residency, inference_session_kv_transfers,
inference_session_kv_transfer_payloads, inference_prompt_cache_entries; plus the ring tables.
Writes go through one process-wide writer lock with retry on ``database is locked`` (the
reference's single-writer gate and lock retry, ``state.rs:148-246``, ``api/error.rs:14-200``).
"""
from __future__ import annotations

import json
import sqlite3
import threading
import time
from contextlib import contextmanager
from pathlib import Path
from typing import Any, Iterable, List, Optional

SCHEMA = """
CREATE TABLE IF NOT EXISTS networks (
  network_id TEXT PRIMARY KEY, name TEXT NOT NULL, owner_device_id TEXT, created_at REAL NOT NULL,
  scheduling_policy TEXT NOT NULL DEFAULT '{}', connectivity TEXT NOT NULL DEFAULT '{}');
CREATE TABLE IF NOT EXISTS devices (
  device_id TEXT PRIMARY KEY, network_id TEXT, name TEXT, public_key TEXT, certificate TEXT,
  tier TEXT NOT NULL DEFAULT 'tier2', cpu_cores INTEGER DEFAULT 0, ram_mb INTEGER DEFAULT 0,
  gpu TEXT DEFAULT '{}', provider TEXT DEFAULT 'cpu', contributed_memory INTEGER DEFAULT 0,
  status TEXT NOT NULL DEFAULT 'online', last_heartbeat REAL, created_at REAL NOT NULL,
  capabilities TEXT DEFAULT '{}', tensor_plane_addr TEXT, throughput_tps REAL DEFAULT 0);
CREATE TABLE IF NOT EXISTS ledger_events (
  event_id TEXT PRIMARY KEY, network_id TEXT, device_id TEXT, job_id TEXT, event_type TEXT NOT NULL,
  credits REAL NOT NULL DEFAULT 0, details TEXT DEFAULT '{}', created_at REAL NOT NULL);
CREATE TABLE IF NOT EXISTS ring_members (
  device_id TEXT PRIMARY KEY, network_id TEXT NOT NULL, model_id TEXT NOT NULL, position INTEGER NOT NULL,
  column_start INTEGER NOT NULL, column_end INTEGER NOT NULL, contributed_memory INTEGER DEFAULT 0,
  status TEXT NOT NULL DEFAULT 'active', joined_at REAL NOT NULL);
CREATE TABLE IF NOT EXISTS ring_state (
  network_id TEXT NOT NULL, model_id TEXT NOT NULL, version INTEGER NOT NULL DEFAULT 0, updated_at REAL,
  PRIMARY KEY (network_id, model_id));
CREATE TABLE IF NOT EXISTS ring_handoffs (
  handoff_id TEXT PRIMARY KEY, network_id TEXT, model_id TEXT, from_device_id TEXT, to_device_id TEXT,
  column_start INTEGER, column_end INTEGER, status TEXT NOT NULL, created_at REAL, updated_at REAL);
CREATE TABLE IF NOT EXISTS ring_callbacks (device_id TEXT PRIMARY KEY, url TEXT NOT NULL, created_at REAL);
CREATE TABLE IF NOT EXISTS inference_jobs (
  job_id TEXT PRIMARY KEY, network_id TEXT NOT NULL, model_id TEXT NOT NULL, submitter_device_id TEXT,
  prompt_tokens TEXT NOT NULL, max_tokens INTEGER NOT NULL, temperature REAL, top_p REAL,
  status TEXT NOT NULL, created_at REAL NOT NULL, updated_at REAL NOT NULL, plan TEXT DEFAULT '{}',
  credits_reserved REAL DEFAULT 0, generated_tokens TEXT, ttft_ms INTEGER, completion_tokens INTEGER DEFAULT 0,
  execution_time_ms INTEGER DEFAULT 0, error TEXT, runtime_mode TEXT DEFAULT 'throughput_first');
CREATE TABLE IF NOT EXISTS inference_sessions (
  session_id TEXT PRIMARY KEY, job_id TEXT NOT NULL, status TEXT NOT NULL, phase TEXT NOT NULL,
  kv_owner_device_id TEXT, kv_seq_len INTEGER DEFAULT 0, created_at REAL, updated_at REAL);
CREATE TABLE IF NOT EXISTS inference_serving_groups (
  group_id TEXT PRIMARY KEY, job_id TEXT NOT NULL, session_id TEXT, phase TEXT NOT NULL,
  member_device_ids TEXT NOT NULL, status TEXT NOT NULL DEFAULT 'planned');
CREATE TABLE IF NOT EXISTS inference_job_assignments (
  assignment_id TEXT PRIMARY KEY, job_id TEXT NOT NULL, session_id TEXT, device_id TEXT NOT NULL,
  phase TEXT NOT NULL, segment_id TEXT, group_id TEXT, status TEXT NOT NULL, lease_id TEXT,
  lease_expires REAL, shard_column_start INTEGER, shard_column_end INTEGER, worker_position INTEGER,
  total_workers INTEGER, created_at REAL, updated_at REAL, execution_time_ms INTEGER DEFAULT 0);
CREATE TABLE IF NOT EXISTS inference_decode_queue (
  session_id TEXT PRIMARY KEY, job_id TEXT NOT NULL, network_id TEXT, status TEXT NOT NULL,
  lease_id TEXT, lease_device_id TEXT, lease_expires REAL, decode_steps_served INTEGER DEFAULT 0,
  fairness_epoch INTEGER DEFAULT 0, kv_seq_len INTEGER DEFAULT 0, updated_at REAL);
CREATE TABLE IF NOT EXISTS inference_decode_batch_events (
  id INTEGER PRIMARY KEY AUTOINCREMENT, network_id TEXT, device_id TEXT, batch_size INTEGER,
  kv_tokens INTEGER, created_at REAL);
CREATE TABLE IF NOT EXISTS inference_scheduler_events (
  id INTEGER PRIMARY KEY AUTOINCREMENT, network_id TEXT, job_id TEXT, event TEXT, details TEXT, created_at REAL);
CREATE TABLE IF NOT EXISTS inference_regroup_events (
  id INTEGER PRIMARY KEY AUTOINCREMENT, job_id TEXT, session_id TEXT, decision TEXT, details TEXT, created_at REAL);
CREATE TABLE IF NOT EXISTS inference_session_checkpoints (
  job_id TEXT NOT NULL, session_id TEXT NOT NULL, payload BLOB NOT NULL, token_index INTEGER, created_at REAL,
  source_device_id TEXT, PRIMARY KEY (job_id, session_id));
CREATE TABLE IF NOT EXISTS inference_session_kv_residency (
  session_id TEXT NOT NULL, device_id TEXT NOT NULL, seq_len INTEGER, updated_at REAL,
  PRIMARY KEY (session_id, device_id));
CREATE TABLE IF NOT EXISTS inference_session_kv_transfers (
  transfer_id TEXT PRIMARY KEY, job_id TEXT, session_id TEXT, source_device_id TEXT, target_device_id TEXT,
  status TEXT NOT NULL, created_at REAL, updated_at REAL);
CREATE TABLE IF NOT EXISTS inference_session_kv_transfer_payloads (
  transfer_id TEXT PRIMARY KEY, payload BLOB NOT NULL, created_at REAL);
CREATE TABLE IF NOT EXISTS inference_prompt_cache_entries (
  prefix_hash TEXT NOT NULL, model_id TEXT NOT NULL, device_id TEXT, tokens INTEGER, created_at REAL,
  PRIMARY KEY (prefix_hash, model_id));
"""


class DbLocked(RuntimeError):
    """Raised when the writer lock could not be taken in time (HTTP 503 + x-meshnet-db-locked)."""


class Database:
    def __init__(self, path: str = ":memory:", lock_timeout_s: float = 10.0):
        self.path = path
        self.lock_timeout_s = lock_timeout_s
        self._conn = sqlite3.connect(path, check_same_thread=False, isolation_level=None, timeout=lock_timeout_s)
        self._conn.row_factory = sqlite3.Row
        if path != ":memory:":
            self._conn.execute("PRAGMA journal_mode=WAL")
        self._conn.execute("PRAGMA foreign_keys=ON")
        self._writer = threading.RLock()
        self._conn.executescript(SCHEMA)

    @contextmanager
    def tx(self):
        """IMMEDIATE transaction under the writer lock; retries ``database is locked`` with 100 ms
        steps up to the lock timeout."""
        if not self._writer.acquire(timeout=self.lock_timeout_s):
            raise DbLocked("database writer lock timed out")
        try:
            deadline = time.monotonic() + self.lock_timeout_s
            while True:
                try:
                    self._conn.execute("BEGIN IMMEDIATE")
                    break
                except sqlite3.OperationalError as e:
                    if "locked" not in str(e) or time.monotonic() > deadline:
                        raise DbLocked(str(e)) from e
                    time.sleep(0.1)
            try:
                yield self._conn
                self._conn.execute("COMMIT")
            except BaseException:
                self._conn.execute("ROLLBACK")
                raise
        finally:
            self._writer.release()

    def query(self, sql: str, args: Iterable[Any] = ()) -> List[dict]:
        with self._writer:
            return [dict(r) for r in self._conn.execute(sql, tuple(args)).fetchall()]

    def one(self, sql: str, args: Iterable[Any] = ()) -> Optional[dict]:
        rows = self.query(sql, args)
        return rows[0] if rows else None


def dumps(x) -> str:
    return json.dumps(x, sort_keys=True)


def loads(s: Optional[str], default=None):
    if s is None:
        return default
    return json.loads(s)
