"""HTTP client of the control-plane API (the reference agent's ``api/registration.rs``)."""
from __future__ import annotations

from typing import List, Optional

import requests


class ControlPlaneClient:
    def __init__(self, base_url: str = "http://localhost:8080", timeout_s: float = 30.0):
        self.base = base_url.rstrip("/")
        self.timeout = timeout_s
        self.s = requests.Session()

    def _req(self, method, path, retries: int = 20, **kw):
        for attempt in range(retries):
            r = self.s.request(method, self.base + path, timeout=self.timeout, **kw)
            if r.status_code == 503 and r.headers.get("x-meshnet-db-locked"):
                import time
                time.sleep(0.1 * (attempt + 1))
                continue
            if r.status_code >= 400:
                raise RuntimeError(f"{method} {path} -> {r.status_code}: {r.text}")
            return r.json()
        raise RuntimeError(f"{method} {path}: database stayed locked")

    def health(self):
        return self._req("GET", "/health")

    def create_network(self, name, owner_device_id=None):
        return self._req("POST", "/api/networks", json={"name": name, "owner_device_id": owner_device_id})

    def list_networks(self):
        return self._req("GET", "/api/networks")

    def register(self, **kw):
        return self._req("POST", "/api/devices/register", json=kw)

    def heartbeat(self, device_id, throughput_tps=None):
        return self._req("POST", f"/api/devices/{device_id}/heartbeat", json={"throughput_tps": throughput_tps})

    def join_ring(self, device_id, network_id, model_id, contributed_memory=0):
        return self._req("POST", "/api/ring/join", json=dict(device_id=device_id, network_id=network_id,
                                                             model_id=model_id, contributed_memory=contributed_memory))

    def leave_ring(self, device_id):
        return self._req("DELETE", f"/api/ring/leave/{device_id}")

    def topology(self, network_id, model_id=None):
        p = {"network_id": network_id}
        if model_id:
            p["model_id"] = model_id
        return self._req("GET", "/api/ring/topology", params=p)

    def submit(self, network_id, model_id, prompt=None, prompt_tokens=None, max_tokens=100, temperature=0.7, top_p=0.9,
               submitter_device_id=None):
        return self._req("POST", "/api/inference/submit", json=dict(
            network_id=network_id, model_id=model_id, prompt=prompt, prompt_tokens=prompt_tokens, max_tokens=max_tokens,
            temperature=temperature, top_p=top_p, submitter_device_id=submitter_device_id))

    def claim(self, device_id, max_decode_sessions=64):
        return self._req("POST", "/api/inference/assignments/claim",
                         json={"device_id": device_id, "max_decode_sessions": max_decode_sessions})

    def ack(self, job_id, device_id):
        return self._req("POST", f"/api/inference/jobs/{job_id}/ack", json={"device_id": device_id})

    def progress(self, job_id, **kw):
        return self._req("POST", f"/api/inference/jobs/{job_id}/progress", json=kw)

    def result(self, job_id, **kw):
        return self._req("POST", f"/api/inference/jobs/{job_id}/result", json=kw)

    def renew(self, lease_id):
        return self._req("POST", f"/api/inference/decode/leases/{lease_id}/renew")

    def release(self, lease_id, session_ids: Optional[List[str]] = None):
        return self._req("POST", f"/api/inference/decode/leases/{lease_id}/release", json={"session_ids": session_ids})

    def upload_checkpoint(self, job_id, session_id, payload: bytes, token_index=0):
        return self._req("POST", f"/api/inference/jobs/{job_id}/session-checkpoints",
                         json={"session_id": session_id, "payload_hex": payload.hex(), "token_index": token_index})

    def download_checkpoint(self, job_id, session_id) -> bytes:
        return bytes.fromhex(self._req("GET", f"/api/inference/jobs/{job_id}/session-checkpoints/{session_id}")
                             ["payload_hex"])

    def job(self, job_id):
        return self._req("GET", f"/api/inference/jobs/{job_id}")

    def cancel(self, job_id):
        return self._req("DELETE", f"/api/inference/jobs/{job_id}")

    def decode_queue(self, network_id=None):
        return self._req("GET", "/api/inference/decode/queue", params={"network_id": network_id} if network_id else {})

    def scheduler_status(self, network_id):
        return self._req("GET", f"/api/status/networks/{network_id}/scheduler")

    def ledger_summary(self, network_id=None):
        return self._req("GET", "/api/ledger/summary", params={"network_id": network_id} if network_id else {})

    def ledger_events(self, network_id=None, device_id=None, limit=100):
        p = {"limit": limit}
        if network_id:
            p["network_id"] = network_id
        if device_id:
            p["device_id"] = device_id
        return self._req("GET", "/api/ledger/events", params=p)
