"""The local device API (``mesh ui``) against a live control plane, on CPU: every route answers,
and each one agrees with the CLI command behind it."""
import socket
import threading
import time

import pytest
from fastapi.testclient import TestClient


@pytest.fixture()
def control_plane():
    import uvicorn
    from mesh_b200.control_plane.app import create_app
    from mesh_b200.control_plane.db import Database
    from mesh_b200.control_plane.service import ControlPlane
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    cp = ControlPlane(Database())
    srv = uvicorn.Server(uvicorn.Config(create_app(cp, presence_interval_s=0), host="127.0.0.1", port=port,
                                        log_level="error"))
    th = threading.Thread(target=srv.run, daemon=True)
    th.start()
    while not srv.started:
        time.sleep(0.05)
    yield cp, f"http://127.0.0.1:{port}"
    srv.should_exit = True
    th.join(timeout=5)


def test_local_api_routes(tmp_path, monkeypatch, control_plane):
    from mesh_b200.cli.local_api import create_local_app
    cp, url = control_plane
    monkeypatch.setenv("MESHNET_HOME", str(tmp_path))
    api = TestClient(create_local_app())
    assert api.get("/health").text == "ok"
    dash = api.get("/api/local/dashboard").json()
    assert dash["device"]["initialised"] is False and dash["runtime"]["running"] is False
    net = cp.create_network("lan")["network_id"]
    r = api.post("/api/local/device/init", json={"network_id": net, "control_plane": url, "preferred_provider": "cpu",
                                                 "device_id": "dev-ui"})
    assert r.status_code == 200, r.text
    st = api.get("/api/local/device/status").json()
    assert st["device_id"] == "dev-ui" and "private_key" not in st and st["runtime"]["running"] is False
    assert st["shards"]["shards"] == {} and st["resources"]["locked"] is False

    # resources: lock records the commitment, unlock is refused inside the cooldown
    r = api.post("/api/local/resource/lock", json={"memory": "1GB"})
    assert r.status_code == 200, r.text
    assert r.json()["locked"] and r.json()["user_allocated"] == 10 ** 9
    assert api.get("/api/local/resource/status").json()["locked_memory"] == int(1.07 * 10 ** 9)
    r = api.post("/api/local/resource/unlock")
    assert r.status_code == 400 and "cooldown active: 24 hours" in r.json()["detail"]
    assert api.post("/api/local/resource/lock", json={"memory": "1GB"}).status_code == 400  # already locked

    # ring
    assert api.post("/api/local/ring/join", json={"model_id": "tiny"}).status_code == 200
    assert api.get("/api/local/ring/status").json()["total_workers"] == 1
    assert api.get("/api/local/ring/shard").json()["column_end"] == 512
    assert api.get("/api/local/ring/topology").json()["workers"][0]["device_id"] == "dev-ui"

    # jobs
    job = api.post("/api/local/jobs", json={"prompt": "hello", "model_id": "tiny", "max_tokens": 3,
                                            "temperature": 0}).json()
    assert job["status"] == "pending" and job["quote"]["total_credits"] > 0
    got = api.get(f"/api/local/jobs/{job['job_id']}").json()
    assert got["job_id"] == job["job_id"]
    assert api.delete(f"/api/local/jobs/{job['job_id']}").status_code == 200
    assert api.get(f"/api/local/jobs/{job['job_id']}").json()["status"] == "cancelled"
    assert api.get("/api/local/jobs/not-a-job").status_code == 400
    assert isinstance(api.get("/api/local/jobs/stats").json(), dict)

    # ledger, pools, doctor, quote
    assert "earned" in api.get("/api/local/ledger/summary").json()
    assert isinstance(api.get("/api/local/ledger/events", params={"limit": 5}).json(), list)
    pool = api.post("/api/local/pools", json={"name": "lab"}).json()
    assert [p["pool_id"] for p in api.get("/api/local/pools").json()] == [pool["pool_id"]]
    assert api.get(f"/api/local/pools/{pool['pool_id']}/status").json()["peer_count"] == 0
    assert api.get(f"/api/local/pools/{pool['pool_id']}/peers").json() == []
    assert api.get("/api/local/pools/nope/status").status_code == 404
    doc = api.post("/api/local/doctor", json={"stage": "preflight"}).json()
    assert {"python", "torch"} <= {c["check"] for c in doc["checks"]}
    q = api.get("/api/local/models/llama3-8b/quote", params={"prompt_tokens": 100, "max_tokens": 50}).json()
    assert q["total_credits"] == q["prompt_credits"] + q["completion_credits"] and q["model_size_factor"] >= 1
    assert api.get("/api/local/models/no-such-model/quote").status_code == 404
    dash = api.get("/api/local/dashboard").json()
    assert dash["device"]["device_id"] == "dev-ui" and dash["ring"]["total_workers"] == 1
    assert api.post("/api/local/device/stop").json()["stopped"] is False
    assert api.post("/api/local/ring/leave").status_code == 200
