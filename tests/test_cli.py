"""The mesh CLI against a live control plane (CPU)."""
import json
import os
import threading
import time

import pytest

from mesh_b200.cli import main as cli


def test_cli_device_ring_job_ledger_pool(tmp_path, monkeypatch, capsys):
    import socket
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
    try:
        monkeypatch.setenv("MESHNET_HOME", str(tmp_path))
        net = cp.create_network("lan")["network_id"]
        url = f"http://127.0.0.1:{port}"
        assert cli.main(["device", "init", "-n", net, "-c", url, "--preferred-provider", "cpu",
                         "--device-id", "dev-a"]) == 0
        assert (tmp_path / "device.toml").exists()
        dev = cli.load_device()  # the control plane issued a certificate for this device's key
        assert dev["certificate"] and dev["control_plane_public_key"] == cp.keypair.public_key().hex()
        assert cli.main(["resource", "lock", "-m", "2G"]) == 0
        assert cli.main(["ring", "join", "-m", "tiny"]) == 0
        capsys.readouterr()
        assert cli.main(["ring", "shard"]) == 0
        shard = json.loads(capsys.readouterr().out)
        assert shard["column_start"] == 0 and shard["column_end"] == 512
        assert cli.main(["job", "run", "-p", "hello", "-m", "tiny", "-n", "3", "-t", "0"]) == 0
        job = json.loads(capsys.readouterr().out)
        assert job["status"] == "pending"
        # run the worker loop of this device in-process for a few rounds
        from mesh_b200.runtime.worker import Worker
        d = cli.load_device()
        w = Worker(cli.client(d), d["device_id"], d["network_id"], "tiny", cli.build_coordinator(d, "tiny"),
                   heartbeat_interval_s=0.2)
        w.start()
        for _ in range(3):
            w.run_once()
        assert cli.main(["job", "status", "--job-id", job["job_id"]]) == 0
        st = json.loads(capsys.readouterr().out)
        assert st["status"] == "completed" and len(st["generated_tokens"]) == 3
        assert cli.main(["ledger", "summary"]) == 0
        assert "dev-a" in json.loads(capsys.readouterr().out)["earned"]
        assert cli.main(["pool", "create", "-n", "p"]) == 0
        pid = json.loads(capsys.readouterr().out)["pool_id"]
        assert cli.main(["pool", "list"]) == 0
        assert json.loads(capsys.readouterr().out)[0]["pool_id"] == pid
        w.stop()
    finally:
        srv.should_exit = True
        th.join(timeout=5)


def test_cli_doctor_preflight_runs(capsys):
    rc = cli.main(["doctor", "--stage", "preflight"])
    out = json.loads(capsys.readouterr().out)
    names = {c["check"] for c in out}
    assert {"python", "torch", "kernels_built", "runtime_built"} <= names
    assert rc in (0, 1)


def test_cli_pool_certificates(tmp_path, monkeypatch, capsys):
    """An admin creates a pool and issues a certificate; a second device joins with it, and a
    certificate from another pool is refused."""
    import json
    from mesh_b200.cli import main as cli
    from mesh_b200.net import pki
    admin_home, member_home = tmp_path / "a", tmp_path / "m"
    monkeypatch.setenv("MESHNET_HOME", str(admin_home))
    assert cli.main(["pool", "create", "-n", "lab"]) == 0
    created = json.loads(capsys.readouterr().out)
    member = pki.KeyPair()
    assert cli.main(["pool", "issue", "--pool-id", created["pool_id"], "--device-pubkey", member.public.hex()]) == 0
    cert_file = tmp_path / "cert.json"
    cert_file.write_text(capsys.readouterr().out)
    monkeypatch.setenv("MESHNET_HOME", str(member_home))
    assert cli.main(["pool", "join", "--pool-id", created["pool_id"], "--pool-root-pubkey",
                     created["root_public_key"], "--cert", str(cert_file)]) == 0
    assert json.loads(capsys.readouterr().out)["certified"] is True
    other = pki.MembershipCert.issue(member.public, pki.KeyPair())
    bad = tmp_path / "bad.json"
    bad.write_text(json.dumps(other.to_dict()))
    import pytest
    with pytest.raises(SystemExit):
        cli.main(["pool", "join", "--pool-id", created["pool_id"], "--pool-root-pubkey", created["root_public_key"],
                  "--cert", str(bad)])
