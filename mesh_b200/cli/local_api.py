"""Local device API behind ``mesh ui`` (the route table of ``agent/src/ui.rs:583-612``).

Every route runs the same code as the matching ``mesh`` command, so the API and the CLI cannot
drift apart: a route builds the command line, runs it in-process and returns what it printed
(parsed as JSON where it is JSON) with 200, or its message with 400 when it fails. Reads that have
no command (dashboard, model quote) are built from the same helpers. ``device/start`` runs the
supervisor as a child process of the API server; ``device/stop`` ends that child (by its own PID).
The browser dashboard itself is not shipped.
"""
from __future__ import annotations

import contextlib
import io
import json
import subprocess
import sys
import threading
from typing import List, Optional

from fastapi import Body, FastAPI, HTTPException
from fastapi.responses import PlainTextResponse


def _run(argv: List[str]):
    """Run ``mesh <argv>`` in this process; its printed output, parsed when it is JSON."""
    from . import main as cli
    out, err = io.StringIO(), io.StringIO()
    try:
        with contextlib.redirect_stdout(out), contextlib.redirect_stderr(err):
            rc = cli.main(argv)
    except SystemExit as e:
        rc = e.code if isinstance(e.code, int) else 1
        err.write(str(e.code) if not isinstance(e.code, int) else "")
    except Exception as e:  # a command's own error becomes a 400, not a 500
        raise HTTPException(400, f"{type(e).__name__}: {e}")
    text = out.getvalue().strip()
    if rc not in (0, None):
        raise HTTPException(400, (err.getvalue() or text or f"mesh {' '.join(argv)} exited {rc}").strip())
    try:
        return json.loads(text)
    except ValueError:
        return {"message": text}


def _opt(argv: List[str], flag: str, value) -> List[str]:
    return argv + [flag, str(value)] if value not in (None, "") else argv


class _Supervisor:
    def __init__(self):
        self.proc: Optional[subprocess.Popen] = None
        self.lock = threading.Lock()

    def start(self, log_level: str):
        with self.lock:
            if self.proc is not None and self.proc.poll() is None:
                raise HTTPException(409, f"device runtime already running (pid {self.proc.pid})")
            self.proc = subprocess.Popen([sys.executable, "-m", "mesh_b200.cli", "device", "start",
                                          "--log-level", log_level])
            return {"started": True, "pid": self.proc.pid}

    def stop(self):
        with self.lock:
            if self.proc is None or self.proc.poll() is not None:
                return {"stopped": False, "message": "device runtime is not running"}
            self.proc.terminate()
            try:
                self.proc.wait(timeout=10)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.proc.wait(timeout=10)
            return {"stopped": True, "returncode": self.proc.returncode}

    def status(self):
        running = self.proc is not None and self.proc.poll() is None
        return {"running": running, "pid": self.proc.pid if running else None}


def create_local_app() -> FastAPI:
    app = FastAPI(title="mesh local api")
    sup = _Supervisor()
    app.state.supervisor = sup

    @app.get("/health", response_class=PlainTextResponse)
    def health():
        return "ok"

    @app.get("/api/local/dashboard")
    def dashboard():
        from . import main as cli
        out = {"device": None, "ring": None, "ledger": None, "runtime": sup.status()}
        try:
            out["device"] = cli.device_status()
        except SystemExit as e:
            out["device"] = {"initialised": False, "message": str(e.code)}
            return out
        for key, argv in (("ring", ["ring", "status"]), ("ledger", ["ledger", "summary"])):
            try:
                out[key] = _run(argv)
            except HTTPException as e:
                out[key] = {"error": e.detail}
        return out

    # ---------------------------------------------------------------- device
    @app.post("/api/local/device/init")
    def device_init(network_id: str = Body(...), name: str = Body("My Device"),
                    control_plane: str = Body("http://localhost:8080"), preferred_provider: Optional[str] = Body(None),
                    device_id: Optional[str] = Body(None), tp: int = Body(1), model_dir: str = Body("")):
        argv = ["device", "init", "-n", network_id, "-d", name, "-c", control_plane, "--tp", str(tp)]
        argv = _opt(_opt(_opt(argv, "--preferred-provider", preferred_provider), "--device-id", device_id),
                    "--model-dir", model_dir)
        return _run(argv)

    @app.post("/api/local/device/start")
    def device_start(log_level: str = Body("info", embed=True)):
        return sup.start(log_level)

    @app.post("/api/local/device/stop")
    def device_stop():
        return sup.stop()

    @app.get("/api/local/device/status")
    def device_status():
        return {**_run(["device", "status"]), "runtime": sup.status()}

    # ---------------------------------------------------------------- resources
    @app.post("/api/local/resource/lock")
    def resource_lock(memory: str = Body(..., embed=True)):
        _run(["resource", "lock", "-m", memory])
        return _run(["resource", "status"])

    @app.post("/api/local/resource/unlock")
    def resource_unlock():
        return _run(["resource", "unlock"])

    @app.get("/api/local/resource/status")
    def resource_status():
        return _run(["resource", "status"])

    # ---------------------------------------------------------------- ring
    @app.post("/api/local/ring/join")
    def ring_join(model_id: str = Body(...), memory: Optional[str] = Body(None)):
        return _run(_opt(["ring", "join", "-m", model_id], "-M", memory))

    @app.post("/api/local/ring/leave")
    def ring_leave():
        return _run(["ring", "leave"])

    @app.get("/api/local/ring/status")
    def ring_status():
        return _run(["ring", "status"])

    @app.get("/api/local/ring/topology")
    def ring_topology():
        return _run(["ring", "topology"])

    @app.get("/api/local/ring/shard")
    def ring_shard():
        return _run(["ring", "shard"])

    # ---------------------------------------------------------------- jobs
    @app.post("/api/local/jobs")
    def submit_job(prompt: str = Body(...), model_id: str = Body("tinyllama-1.1b"), max_tokens: int = Body(100),
                   temperature: float = Body(1.0), top_p: float = Body(0.9)):
        return _run(["job", "run", "-p", prompt, "-m", model_id, "-n", str(max_tokens), "-t", str(temperature),
                     "--top-p", str(top_p)])

    @app.get("/api/local/jobs/stats")
    def job_stats():
        return _run(["job", "stats"])

    @app.get("/api/local/jobs/{job_id}")
    def job_status(job_id: str):
        return _run(["job", "status", "--job-id", job_id])

    @app.delete("/api/local/jobs/{job_id}")
    def cancel_job(job_id: str):
        from . import main as cli
        try:
            return cli.client(cli.load_device()).cancel(job_id)
        except Exception as e:
            raise HTTPException(400, f"{type(e).__name__}: {e}")

    # ---------------------------------------------------------------- ledger
    @app.get("/api/local/ledger/summary")
    def ledger_summary(job_id: Optional[str] = None):
        return _run(_opt(["ledger", "summary"], "--job-id", job_id))

    @app.get("/api/local/ledger/events")
    def ledger_events(job_id: Optional[str] = None, limit: int = 20):
        return _run(_opt(["ledger", "events", "--limit", str(limit)], "--job-id", job_id))

    # ---------------------------------------------------------------- pools
    @app.get("/api/local/pools")
    def list_pools():
        return _run(["pool", "list"])

    @app.post("/api/local/pools")
    def create_pool(name: str = Body(..., embed=True)):
        return _run(["pool", "create", "-n", name])

    @app.post("/api/local/pools/join")
    def join_pool(pool_id: str = Body(...), pool_root_pubkey: str = Body(...), name: Optional[str] = Body(None),
                  cert: Optional[str] = Body(None)):
        argv = ["pool", "join", "--pool-id", pool_id, "--pool-root-pubkey", pool_root_pubkey]
        return _run(_opt(_opt(argv, "-n", name), "--cert", cert))

    @app.get("/api/local/pools/{pool_id}/peers")
    def pool_peers(pool_id: str):
        return _run(["pool", "peers", "--pool-id", pool_id])

    @app.get("/api/local/pools/{pool_id}/status")
    def pool_status(pool_id: str):
        mine = [p for p in _run(["pool", "list"]) if p.get("pool_id") == pool_id]
        if not mine:
            raise HTTPException(404, f"pool {pool_id} is not known to this device")
        p = mine[0]
        return {**p, "peer_count": len(p.get("peers", []))}

    # ---------------------------------------------------------------- doctor, models
    @app.post("/api/local/doctor")
    def doctor(stage: str = Body("production", embed=True)):
        from . import main as cli
        out = io.StringIO()
        with contextlib.redirect_stdout(out):
            rc = cli.main(["doctor", "--stage", stage])
        return {"ok": rc == 0, "checks": json.loads(out.getvalue())}

    @app.get("/api/local/models/{model_id}/quote")
    def model_quote(model_id: str, prompt_tokens: int = 128, max_tokens: int = 256):
        from ..config import get_preset
        from ..control_plane import policy
        try:
            cfg = get_preset(model_id)
        except (KeyError, ValueError):
            raise HTTPException(404, f"unknown model {model_id}")
        total = int(cfg.param_count() * 4)
        return {"model_id": model_id, "total_model_bytes": total,
                **policy.consumption(prompt_tokens, max_tokens, total)}

    return app
