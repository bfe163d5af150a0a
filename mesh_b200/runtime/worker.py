"""Worker runtime: the ``mesh device runtime`` loop of one ring member.

Restates ``agent/src/main.rs:3629-4787`` (``cmd_runtime``): register, heartbeat thread, join the
ring, then loop: claim work; a prefill assignment runs the prefill segment, reports
PrefillComplete progress and uploads a session checkpoint (so any decode group member can resume
it); a decode lease runs the cohort's sessions to completion with microbatching, renewing the
lease and reporting progress every ``progress_report_interval`` tokens, then reports results.
On an execution error the lease is released so the sessions can be retried elsewhere
(``main.rs:2752-2767``). Idle polls sleep 1 s, active decode ticks 10 ms.
"""
from __future__ import annotations

import threading
import time
import traceback
from typing import Optional

from ..engine.coordinator import InferenceCoordinator
from ..engine.types import ExecutionPhase, GenerationConfig, InferenceRequest, PrefillComplete
from .client import ControlPlaneClient


class Worker:
    def __init__(self, client: ControlPlaneClient, device_id: str, network_id: str, model_id: str, coordinator:
                 InferenceCoordinator, tier: str = "tier2", provider: str = "cpu", contributed_memory: int = 0,
                 heartbeat_interval_s: float = 5.0, idle_sleep_s: float = 1.0):
        self.c = client
        self.device_id = device_id
        self.network_id = network_id
        self.model_id = model_id
        self.coord = coordinator
        self.tier, self.provider, self.mem = tier, provider, contributed_memory
        self.hb_interval = heartbeat_interval_s
        self.idle_sleep = idle_sleep_s
        self._stop = threading.Event()
        self.completed = 0

    def start(self):
        self.c.register(device_id=self.device_id, network_id=self.network_id, name=self.device_id, tier=self.tier,
                        provider=self.provider, contributed_memory=self.mem)
        self.c.join_ring(self.device_id, self.network_id, self.model_id, self.mem)
        threading.Thread(target=self._heartbeat, daemon=True, name=f"hb-{self.device_id}").start()

    def stop(self):
        self._stop.set()

    def _heartbeat(self):
        while not self._stop.wait(self.hb_interval):
            try:
                tps = self.coord.stats.derived()["avg_tokens_per_second"]
                self.c.heartbeat(self.device_id, tps)
            except Exception:
                pass

    def _request(self, a: dict, phase: ExecutionPhase) -> InferenceRequest:
        return InferenceRequest(network_id=self.network_id, model_id=a["model_id"], prompt_tokens=a["prompt_tokens"],
                                executor_id=self.device_id, job_id=a["job_id"], session_id=a["session_id"],
                                phase=phase, config=GenerationConfig(max_tokens=a["max_tokens"],
                                                                     temperature=a["temperature"], top_p=a["top_p"]))

    def run_once(self) -> str:
        """One claim/execute/report round; returns the kind of work done."""
        w = self.c.claim(self.device_id)
        kind = w["kind"]
        if kind == "prefill":
            for a in w["assignments"]:
                self.c.ack(a["job_id"], self.device_id)
                req = self._request(a, ExecutionPhase.PREFILL)
                try:
                    pc: PrefillComplete = self.coord.process_segment(req)
                    blob = self.coord.export_session_checkpoint_bytes(req.session_id)
                    self.c.upload_checkpoint(req.job_id, req.session_id, blob, pc.completion_tokens)
                    self.c.progress(req.job_id, device_id=self.device_id, phase="prefill",
                                    completion_tokens=pc.completion_tokens, kv_cache_seq_len=pc.kv_cache_seq_len,
                                    time_to_first_token_ms=pc.time_to_first_token_ms,
                                    execution_time_ms=pc.execution_time_ms)
                except Exception as e:
                    self.c.result(req.job_id, device_id=self.device_id, success=False,
                                  error=f"prefill failed: {e}\n{traceback.format_exc()}")
        elif kind == "decode":
            lease = w["lease_id"]
            reqs = []
            try:
                for a in w["assignments"]:
                    req = self._request(a, ExecutionPhase.DECODE)
                    if req.session_id not in self.coord.sessions:
                        self.coord.hydrate_session(self.c.download_checkpoint(req.job_id, req.session_id))
                    reqs.append(req)
                last_renew = time.monotonic()
                pending = {r.session_id: r for r in reqs}
                while pending:
                    for res in self.coord.step():
                        r = next((x for x in reqs if x.job_id == res.job_id), None)
                        if r is None:
                            continue
                        pending.pop(r.session_id, None)
                        self.c.result(res.job_id, device_id=self.device_id, success=res.success,
                                      generated_tokens=res.generated_tokens, error=res.error,
                                      completion_tokens=res.completion_tokens, execution_time_ms=res.execution_time_ms,
                                      time_to_first_token_ms=res.time_to_first_token_ms)
                        self.completed += 1
                    for sid, r in pending.items():
                        s = self.coord.sessions.get(sid)
                        if s is not None and len(s.generated) % max(r.config.progress_report_interval, 1) == 0:
                            self.c.progress(r.job_id, device_id=self.device_id, phase="decode",
                                            completion_tokens=len(s.generated), kv_cache_seq_len=s.kv_tokens)
                    if time.monotonic() - last_renew > 20.0:
                        self.c.renew(lease)
                        last_renew = time.monotonic()
            except Exception:
                self.c.release(lease, [r.session_id for r in reqs])
                raise
        return kind

    def run(self, max_rounds: Optional[int] = None):
        n = 0
        while not self._stop.is_set() and (max_rounds is None or n < max_rounds):
            kind = self.run_once()
            n += 1
            if kind == "idle":
                self._stop.wait(self.idle_sleep)
