"""HTTP API of the control plane (FastAPI), with the reference's routes
(``control-plane/src/api/mod.rs:314-443``). Binary payloads (checkpoints, KV transfers) travel
hex-encoded in JSON as in the reference. ``python -m mesh_b200.control_plane.app --port 8080``
serves it (the ``mesh-control-plane`` binary of the reference).
"""
from __future__ import annotations

import argparse
import os
import threading
import time
from typing import List, Optional

from fastapi import Body, FastAPI, Request
from fastapi.responses import JSONResponse
from pydantic import BaseModel

from .db import Database, DbLocked
from .service import ApiError, ControlPlane


class NetworkIn(BaseModel):
    name: str
    owner_device_id: Optional[str] = None
    scheduling_policy: Optional[dict] = None


class RegisterIn(BaseModel):
    device_id: str
    network_id: Optional[str] = None
    name: str = ""
    tier: str = "tier2"
    provider: str = "cpu"
    contributed_memory: int = 0
    capabilities: Optional[dict] = None
    public_key: str = ""
    certificate: str = ""
    tensor_plane_addr: str = ""


class HeartbeatIn(BaseModel):
    throughput_tps: Optional[float] = None


class JoinIn(BaseModel):
    device_id: str
    network_id: str
    model_id: str
    contributed_memory: int = 0


class SubmitIn(BaseModel):
    network_id: str
    model_id: str
    prompt: Optional[str] = None
    prompt_tokens: Optional[List[int]] = None
    max_tokens: int = 100
    temperature: float = 0.7
    top_p: float = 0.9
    submitter_device_id: Optional[str] = None
    runtime_mode: str = "throughput_first"


class ClaimIn(BaseModel):
    device_id: str
    max_decode_sessions: int = 64


class ProgressIn(BaseModel):
    device_id: str
    phase: str
    completion_tokens: int = 0
    kv_cache_seq_len: int = 0
    time_to_first_token_ms: Optional[int] = None
    execution_time_ms: int = 0
    kv_transfer: bool = False


class ResultIn(BaseModel):
    device_id: str
    success: bool
    generated_tokens: Optional[List[int]] = None
    error: Optional[str] = None
    completion_tokens: int = 0
    execution_time_ms: int = 0
    time_to_first_token_ms: Optional[int] = None


class CheckpointIn(BaseModel):
    session_id: str
    payload_hex: str
    token_index: int = 0


class KvTransferIn(BaseModel):
    session_id: str
    source_device_id: str
    target_device_id: str
    status: str = "pending"
    transfer_id: Optional[str] = None


class PayloadIn(BaseModel):
    transfer_id: str
    payload_hex: str


class HandoffIn(BaseModel):
    network_id: str
    model_id: str
    from_device_id: str
    to_device_id: str
    column_start: int
    column_end: int


class LedgerIn(BaseModel):
    network_id: str
    device_id: str
    event_type: str
    credits: float = 0.0
    job_id: Optional[str] = None
    details: Optional[dict] = None


def create_app(cp: Optional[ControlPlane] = None, presence_interval_s: Optional[float] = None) -> FastAPI:
    cp = cp or ControlPlane(Database(os.environ.get("MESHNET_CONTROL_PLANE_DB", ":memory:")),
                            model_store=os.environ.get("MESHNET_MODEL_STORE"))
    app = FastAPI(title="mesh_b200 control plane")
    app.state.cp = cp

    @app.exception_handler(ApiError)
    async def _api_error(_req: Request, exc: ApiError):
        return JSONResponse({"error": str(exc)}, status_code=exc.status)

    @app.exception_handler(DbLocked)
    async def _locked(_req: Request, exc: DbLocked):
        return JSONResponse({"error": str(exc)}, status_code=503, headers={"x-meshnet-db-locked": "true"})

    @app.get("/health")
    def health():
        return {"status": "ok"}

    @app.post("/api/networks")
    def create_network(b: NetworkIn):
        return cp.create_network(b.name, b.owner_device_id, b.scheduling_policy)

    @app.get("/api/networks")
    def list_networks():
        return cp.list_networks()

    @app.get("/api/status/networks/{network_id}/scheduler")
    def net_status(network_id: str):
        return cp.network_scheduler_status(network_id)

    @app.get("/api/status/jobs/{job_id}/scheduler")
    def job_sched(job_id: str):
        return cp.job_scheduler_status(job_id)

    @app.post("/api/devices/register")
    def register(b: RegisterIn):
        return cp.register_device(**b.model_dump())

    @app.post("/api/devices/{device_id}/heartbeat")
    def heartbeat(device_id: str, b: HeartbeatIn = Body(default=HeartbeatIn())):
        return cp.heartbeat(device_id, b.throughput_tps)

    @app.post("/api/ledger/events")
    def ledger_event(b: LedgerIn):
        return cp.create_ledger_event(b.network_id, b.device_id, b.event_type, b.credits, b.job_id, b.details)

    @app.get("/api/ledger/events")
    def ledger_events(network_id: Optional[str] = None, device_id: Optional[str] = None, limit: int = 100):
        return cp.list_ledger_events(network_id, device_id, limit)

    @app.get("/api/ledger/summary")
    def ledger_summary(network_id: Optional[str] = None):
        return cp.ledger_summary(network_id)

    @app.post("/api/ring/join")
    def join(b: JoinIn):
        return cp.join_ring(b.device_id, b.network_id, b.model_id, b.contributed_memory)

    @app.get("/api/ring/topology")
    def topology(network_id: str, model_id: Optional[str] = None):
        return cp.topology(network_id, model_id)

    @app.delete("/api/ring/leave/{device_id}")
    def leave(device_id: str):
        return cp.leave_ring(device_id)

    @app.post("/api/ring/handoff")
    def handoff(b: HandoffIn):
        return cp.create_handoff(**b.model_dump())

    @app.get("/api/ring/handoff/{hid}")
    def get_handoff(hid: str):
        return cp.get_handoff(hid)

    @app.patch("/api/ring/handoff/{hid}")
    def patch_handoff(hid: str, body: dict = Body(...)):
        return cp.update_handoff(hid, body.get("status", ""))

    @app.delete("/api/ring/handoff/{hid}")
    def cancel_handoff(hid: str):
        return cp.update_handoff(hid, "cancelled")

    @app.get("/api/ring/handoffs")
    def handoffs(network_id: Optional[str] = None):
        return cp.list_handoffs(network_id)

    @app.post("/api/ring/callback")
    def callback(body: dict = Body(...)):
        return cp.register_callback(body["device_id"], body["url"])

    @app.delete("/api/ring/callback/{device_id}")
    def uncallback(device_id: str):
        return cp.unregister_callback(device_id)

    @app.post("/api/ring/version")
    def version(body: dict = Body(...)):
        return cp.check_topology_version(body["network_id"], body["model_id"], int(body.get("version", 0)))

    @app.post("/api/inference/submit")
    def submit(b: SubmitIn):
        return cp.submit_inference(**b.model_dump())

    @app.post("/api/inference/assignments/claim")
    def claim(b: ClaimIn):
        return cp.claim(b.device_id, b.max_decode_sessions)

    @app.get("/api/inference/decode/queue")
    def decode_queue(network_id: Optional[str] = None):
        return cp.observe_decode_queue(network_id)

    @app.post("/api/inference/decode/leases/{lease_id}/renew")
    def renew(lease_id: str):
        return cp.renew_lease(lease_id)

    @app.post("/api/inference/decode/leases/{lease_id}/release")
    def release(lease_id: str, body: dict = Body(default={})):
        return cp.release_lease(lease_id, body.get("session_ids"))

    @app.post("/api/inference/jobs/{job_id}/ack")
    def ack(job_id: str, body: dict = Body(...)):
        return cp.acknowledge(job_id, body["device_id"])

    @app.post("/api/inference/jobs/{job_id}/result")
    def result(job_id: str, b: ResultIn):
        return cp.report_result(job_id, **b.model_dump())

    @app.post("/api/inference/jobs/{job_id}/progress")
    def progress(job_id: str, b: ProgressIn):
        return cp.report_progress(job_id, **b.model_dump())

    @app.post("/api/inference/jobs/{job_id}/session-checkpoints")
    def up_ckpt(job_id: str, b: CheckpointIn):
        return cp.upload_session_checkpoint(job_id, b.session_id, bytes.fromhex(b.payload_hex), b.token_index)

    @app.get("/api/inference/jobs/{job_id}/session-checkpoints/{session_id}")
    def down_ckpt(job_id: str, session_id: str):
        return {"payload_hex": cp.download_session_checkpoint(job_id, session_id).hex()}

    @app.post("/api/inference/jobs/{job_id}/session-kv-transfers")
    def kv_transfer(job_id: str, b: KvTransferIn):
        return cp.report_kv_transfer(job_id, b.session_id, b.source_device_id, b.target_device_id, b.status,
                                     b.transfer_id)

    @app.get("/api/inference/session-kv-transfers/pending")
    def kv_pending(device_id: str):
        return cp.pending_kv_transfers(device_id)

    @app.post("/api/inference/jobs/{job_id}/session-kv-transfers/payloads")
    def kv_up(job_id: str, b: PayloadIn):
        return cp.upload_kv_payload(b.transfer_id, bytes.fromhex(b.payload_hex))

    @app.get("/api/inference/jobs/{job_id}/session-kv-transfers/{transfer_id}/payload")
    def kv_down(job_id: str, transfer_id: str):
        return {"payload_hex": cp.download_kv_payload(transfer_id).hex()}

    @app.get("/api/inference/jobs/{job_id}")
    def job(job_id: str):
        return cp.job_status(job_id)

    @app.delete("/api/inference/jobs/{job_id}")
    def cancel(job_id: str):
        return cp.cancel_job(job_id)

    if presence_interval_s is None:
        presence_interval_s = float(os.environ.get("MESHNET_PRESENCE_POLL_INTERVAL_MS", "250")) / 1000.0
    if presence_interval_s > 0:
        stop = threading.Event()

        def monitor():
            while not stop.wait(presence_interval_s):
                try:
                    cp.presence_sweep()
                except Exception:
                    pass

        @app.on_event("startup")
        def _start():
            threading.Thread(target=monitor, daemon=True, name="presence-monitor").start()

        @app.on_event("shutdown")
        def _stop():
            stop.set()
    return app


def main():
    ap = argparse.ArgumentParser(prog="mesh-control-plane")
    ap.add_argument("--port", type=int, default=8080)
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--db", default=os.environ.get("MESHNET_CONTROL_PLANE_DB", ""))
    ap.add_argument("--log-level", default="info")
    a = ap.parse_args()
    import uvicorn
    home = os.environ.get("MESHNET_HOME", os.path.expanduser("~/.meshnet"))
    os.makedirs(home, exist_ok=True)
    db = Database(a.db or os.path.join(home, "control_plane.sqlite3"))
    app = create_app(ControlPlane(db, model_store=os.environ.get("MESHNET_MODEL_STORE")))
    uvicorn.run(app, host=a.host, port=a.port, log_level=a.log_level)


if __name__ == "__main__":
    main()
