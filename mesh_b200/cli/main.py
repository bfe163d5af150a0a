"""``mesh`` command line (the reference's ``agent/src/main.rs:299-673`` command tree).

    mesh device init|start|runtime|status       mesh ring join|leave|status|topology|shard
    mesh resource lock|unlock|status            mesh job run|status|watch|stats
    mesh ledger summary|events                  mesh pool create|join|list|peers|status
    mesh model import-hf|reshard|list|info      mesh doctor [--stage preflight|production]
    mesh ui [--api-only]

Device state lives in ``$MESHNET_HOME`` (default ``~/.meshnet``): ``device.toml`` (identity,
control-plane URL, ``[execution]``, ``[governance]`` and the ``[b200]`` section), an ed25519 key,
pools, logs and ``inference_stats.json``.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time
import uuid
from pathlib import Path

try:
    import tomllib
except ImportError:  # pragma: no cover
    tomllib = None


def home() -> Path:
    h = Path(os.environ.get("MESHNET_HOME", str(Path.home() / ".meshnet")))
    h.mkdir(parents=True, exist_ok=True)
    return h


def _toml_value(v):
    if isinstance(v, bool):
        return "true" if v else "false"
    if isinstance(v, (int, float)):
        return repr(v)
    if isinstance(v, list):
        return "[" + ", ".join(_toml_value(x) for x in v) + "]"
    return json.dumps(str(v))


def write_toml(path: Path, data: dict) -> None:
    lines = []
    for k, v in data.items():
        if not isinstance(v, dict):
            lines.append(f"{k} = {_toml_value(v)}")
    for k, v in data.items():
        if isinstance(v, dict):
            lines.append(f"\n[{k}]")
            for kk, vv in v.items():
                lines.append(f"{kk} = {_toml_value(vv)}")
    path.write_text("\n".join(lines) + "\n")


def load_device() -> dict:
    p = home() / "device.toml"
    if not p.exists():
        raise SystemExit("device not initialised: run `mesh device init --network-id <id>` first")
    return tomllib.loads(p.read_text())


def save_device(d: dict) -> None:
    write_toml(home() / "device.toml", d)


def client(d: dict):
    from ..runtime.client import ControlPlaneClient
    return ControlPlaneClient(d.get("control_plane", "http://localhost:8080"))


def gen_keypair() -> tuple:
    """ed25519 device identity (reference ``device/keypair.rs:55-75``)."""
    from cryptography.hazmat.primitives import serialization
    from cryptography.hazmat.primitives.asymmetric.ed25519 import Ed25519PrivateKey
    k = Ed25519PrivateKey.generate()
    priv = k.private_bytes(serialization.Encoding.Raw, serialization.PrivateFormat.Raw,
                           serialization.NoEncryption()).hex()
    pub = k.public_key().public_bytes(serialization.Encoding.Raw, serialization.PublicFormat.Raw).hex()
    return priv, pub


def detect_capabilities() -> dict:
    import psutil
    cap = {"cpu_cores": psutil.cpu_count(logical=True), "ram_mb": psutil.virtual_memory().total // (1 << 20),
           "gpus": []}
    try:
        import torch
        if torch.cuda.is_available():
            for i in range(torch.cuda.device_count()):
                p = torch.cuda.get_device_properties(i)
                cap["gpus"].append({"name": p.name, "memory_mb": p.total_memory // (1 << 20),
                                    "sm": f"{p.major}{p.minor}", "sms": p.multi_processor_count})
    except Exception:
        pass
    ram = cap["ram_mb"]
    gpu_mem = sum(g["memory_mb"] for g in cap["gpus"])
    tier = "tier4" if gpu_mem >= 160_000 else "tier3" if gpu_mem else "tier2" if ram >= 32_000 else "tier1"
    cap["tier"] = tier
    return cap


# ------------------------------------------------------------------------------------------ device
def cmd_device_init(a):
    priv, pub = gen_keypair()
    cap = detect_capabilities()
    d = {"device_id": a.device_id or str(uuid.uuid4()), "name": a.name, "network_id": a.network_id,
         "control_plane": a.control_plane, "public_key": pub, "private_key": priv, "tier": cap["tier"],
         "execution": {"preferred_provider": a.preferred_provider or ("cuda" if cap["gpus"] else "cpu")},
         "governance": {"max_concurrent_jobs": 8, "tensor_plane_max_message_bytes": 10 * 1024 * 1024,
                        "recovery_cooldown_ms": 5000, "recovery_max_loads_per_minute": 8},
         "b200": {"tp": a.tp, "gpu_ids": [g for g in range(len(cap["gpus"]))], "page_tokens": 16,
                  "max_decode_batch": 64, "cuda_graphs": True, "model_dir": a.model_dir or ""}}
    save_device(d)
    try:
        r = client(d).register(device_id=d["device_id"], network_id=a.network_id, name=a.name, tier=cap["tier"],
                               provider=d["execution"]["preferred_provider"], public_key=pub,
                               capabilities=cap)
        if isinstance(r, dict) and r.get("certificate"):
            # keep the certificate the control plane issued, after checking it names this device's key
            from ..control_plane.certificate import verify_certificate
            cert = verify_certificate(bytes.fromhex(r["certificate"]), bytes.fromhex(r["control_plane_public_key"]))
            if cert.public_key.hex() != pub or cert.device_id != d["device_id"]:
                raise SystemExit("the control plane's certificate does not name this device and key")
            d["certificate"] = r["certificate"]
            d["control_plane_public_key"] = r["control_plane_public_key"]
            save_device(d)
        print(f"registered device {d['device_id']} with {a.control_plane}")
    except Exception as e:
        print(f"initialised device {d['device_id']} (control plane unreachable: {e})")


def device_status() -> dict:
    from ..models.registry import ShardRegistry
    d = load_device()
    out = {k: v for k, v in d.items() if k != "private_key"}
    stats = home() / "inference_stats.json"
    if stats.exists():
        out["inference_stats"] = json.loads(stats.read_text())
    rm = resource_manager()
    out["resources"] = rm.status()
    rm.close()
    out["shards"] = ShardRegistry(home() / "shards").summary()
    return out


def cmd_device_status(a):
    print(json.dumps(device_status(), indent=2))


def cmd_device_start(a):
    """Supervisor: run ``mesh device runtime`` as a child and restart it 2 s after an abnormal exit
    (reference ``main.rs:3544-3627``)."""
    restarts = 0
    while True:
        p = subprocess.Popen([sys.executable, "-m", "mesh_b200.cli", "device", "runtime", "--log-level", a.log_level])
        rc = p.wait()
        if rc == 0 or a.no_restart:
            return rc
        restarts += 1
        print(f"runtime exited with {rc}; restarting in 2s (restart {restarts})", file=sys.stderr)
        time.sleep(2.0)


def build_coordinator(d: dict, model_id: str):
    """Backend by preferred provider: the sm_100a engine on cuda, the fp32 oracle on cpu."""
    from ..config import EngineConfig, get_preset
    from ..engine.coordinator import InferenceCoordinator
    from ..engine.stats import InferenceStats
    prov = d.get("execution", {}).get("preferred_provider", "cpu")
    cfg = get_preset(model_id)
    stats = InferenceStats()
    if prov == "cuda":
        import torch
        from ..engine.backend import GpuBackend
        from ..engine.serving import Engine
        from ..models.llama import KVPool, LlamaRunner
        from ..models.weights import synthetic_device_weights
        b2 = d.get("b200", {})
        dev = torch.device("cuda", 0)
        ecfg = EngineConfig(max_seq_len=4096, use_cuda_graphs=b2.get("cuda_graphs", True))
        w = synthetic_device_weights(cfg, 0, 1, device=dev)
        kv = KVPool(cfg, w.layout.local_kv_heads, 4096, b2.get("page_tokens", 16), dev)
        eng = Engine(LlamaRunner(w, ecfg, kv, dev, max_tokens=8192), ecfg, max_batch=b2.get("max_decode_batch", 64))
        return InferenceCoordinator(GpuBackend(eng), ecfg, stats=stats, worker_id=d["device_id"], model_id=model_id)
    from ..engine.backend import CpuReferenceBackend
    from ..models.weights import synthetic_reference_weights
    return InferenceCoordinator(CpuReferenceBackend(synthetic_reference_weights(cfg, seed=0)), EngineConfig(),
                                stats=stats, worker_id=d["device_id"], model_id=model_id)


def _make_worker(d: dict, coord):
    from ..runtime.worker import Worker
    ring = d.get("ring", {})
    return Worker(client(d), d["device_id"], d["network_id"], ring["model_id"], coord, tier=d.get("tier", "tier2"),
                  provider=d.get("execution", {}).get("preferred_provider", "cpu"),
                  contributed_memory=int(ring.get("memory", 0)),
                  heartbeat_interval_s=float(os.environ.get("MESHNET_HEARTBEAT_INTERVAL_MS", "5000")) / 1000.0)


def _tp_group_leader(tb, cfg, ecfg, d=None):
    """Rank 0 of a multi-GPU group: the coordinator over the group backend, driven by the worker loop."""
    from ..engine.coordinator import InferenceCoordinator
    from ..engine.stats import InferenceStats
    stats = InferenceStats()
    coord = InferenceCoordinator(tb, ecfg, stats=stats, worker_id=d["device_id"], model_id=d["ring"]["model_id"])
    w = _make_worker(d, coord)
    w.start()
    try:
        w.run()
    finally:
        stats.save_to_file(str(home()))
    return {"completed": w.completed}


def cmd_device_runtime(a):
    """The long-lived worker: rotating file log, the memory commitment (host commitments pinned
    for the process's life, HBM commitments sizing each GPU's KV pool), the shard registry, then
    the claim loop over one GPU, a TP group of GPUs, or the CPU oracle."""
    import logging
    from ..utils.logs import init_production_logging
    init_production_logging(getattr(a, "log_level", "info"), home() / "logs")
    log = logging.getLogger("mesh.runtime")
    d = load_device()
    ring = d.get("ring", {})
    if not ring.get("model_id"):
        raise SystemExit("join a ring first: `mesh ring join --model-id <id>`")
    rm = resource_manager()
    hbm_commit = rm.cfg.user_allocated if (rm.is_locked and rm.pool == "hbm") else 0
    log.info("resource commitment: %s", rm.status())
    b2 = d.get("b200", {})
    tp = int(b2.get("tp", 1))
    model_dir = b2.get("model_dir") or ""
    try:
        if d.get("execution", {}).get("preferred_provider") == "cuda" and (tp > 1 or model_dir):
            # one process per GPU; rank 0 runs the worker loop and drives the group
            import functools
            import tempfile
            from ..runtime.tp_group import GroupSpec, run_group
            spec = GroupSpec(world=tp, model_dir=model_dir or None, preset=None if model_dir else ring["model_id"],
                             max_seq_len=int(b2.get("max_seq_len", 4096)), num_pages=int(b2.get("kv_pages", 4096)),
                             max_batch=int(b2.get("max_decode_batch", 64)),
                             use_cuda_graphs=bool(b2.get("cuda_graphs", True)),
                             registry_dir=str(home() / "shards"), hbm_commit_bytes=hbm_commit)
            log.info("starting a TP group of %d GPU(s) for %s", tp, ring["model_id"])
            with tempfile.TemporaryDirectory(dir=str(home())) as wd:
                run_group(spec, functools.partial(_tp_group_leader, d=d), wd)
            return
        coord = build_coordinator(d, ring["model_id"])
        w = _make_worker(d, coord)
        w.start()
        try:
            w.run()
        finally:
            coord.stats.save_to_file(str(home()))
    finally:
        rm.close()


# ------------------------------------------------------------------------------------------ resource
def _parse_mem(s: str) -> int:
    from ..runtime.resources import parse_memory_string
    return parse_memory_string(s)


def resource_manager(pool=None):
    from ..runtime.resources import ResourceManager
    return ResourceManager(home() / "resource_lock.toml", pool=pool)


def cmd_resource(a):
    """Commit memory to the mesh (``agent/src/main.rs`` resource commands over the resource
    manager): ``lock`` records the commitment (per-GPU HBM on a GPU box, host RAM otherwise) with
    its cooldown; the device runtime pins host commitments and sizes its KV pool from HBM ones."""
    from ..errors import CooldownActive, MeshError
    d = load_device()
    rm = resource_manager(getattr(a, "pool", None))
    try:
        if a.action == "lock":
            rm.set_allocation(_parse_mem(a.memory))
            rm.lock(pin=False)
            d["resource_lock"] = {"memory_bytes": rm.cfg.user_allocated, "pool": rm.pool,
                                  "locked_at": rm.cfg.lock_timestamp}
            save_device(d)
            print(f"locked {rm.cfg.user_allocated} bytes of {rm.pool} for the mesh "
                  f"({rm.cfg.locked_memory} with the 7% margin); unlock allowed after {rm.cfg.cooldown_hours} h")
        elif a.action == "unlock":
            rm.unlock()
            d.pop("resource_lock", None)
            save_device(d)
            print("unlocked")
        else:
            print(json.dumps(rm.status()))
    except CooldownActive as e:
        print(str(e), file=sys.stderr)
        return 1
    except MeshError as e:
        print(f"resource error: {e}", file=sys.stderr)
        return 1
    finally:
        rm.close()


# ------------------------------------------------------------------------------------------ ring
def cmd_ring(a):
    d = load_device()
    c = client(d)
    if a.action == "join":
        mem = _parse_mem(a.memory) if a.memory else int(d.get("resource_lock", {}).get("memory_bytes", 0))
        t = c.join_ring(d["device_id"], d["network_id"], a.model_id, mem)
        d["ring"] = {"model_id": a.model_id, "memory": mem}
        save_device(d)
        print(json.dumps(t, indent=2))
    elif a.action == "leave":
        print(json.dumps(c.leave_ring(d["device_id"]), indent=2))
        d.pop("ring", None)
        save_device(d)
    elif a.action in ("status", "topology", "shard"):
        t = c.topology(d["network_id"], d.get("ring", {}).get("model_id"))
        if a.action == "shard":
            me = [w for w in t["workers"] if w["device_id"] == d["device_id"]]
            print(json.dumps(me[0] if me else {"member": False}, indent=2))
        elif a.action == "status":
            print(json.dumps({k: t[k] for k in ("version", "total_workers", "stable")}, indent=2))
        else:
            print(json.dumps(t, indent=2))


# ------------------------------------------------------------------------------------------ job
def cmd_job(a):
    d = load_device()
    c = client(d)
    if a.action == "run":
        r = c.submit(d["network_id"], a.model_id, prompt=a.prompt, max_tokens=a.max_tokens,
                     temperature=a.temperature, top_p=a.top_p, submitter_device_id=d["device_id"])
        print(json.dumps({"job_id": r["job_id"], "status": r["status"], "quote": r["quote"]}, indent=2))
        if a.wait:
            _watch(c, r["job_id"], 500)
    elif a.action == "status":
        print(json.dumps(c.job(a.job_id), indent=2, default=str))
    elif a.action == "watch":
        _watch(c, a.job_id, a.interval_ms)
    elif a.action == "stats":
        p = home() / "inference_stats.json"
        print(p.read_text() if p.exists() else "{}")


def _watch(c, job_id, interval_ms):
    while True:
        st = c.job(job_id)
        print(f"{st['status']}: {st.get('completion_tokens', 0)} tokens", flush=True)
        if st["status"] in ("completed", "failed", "cancelled"):
            print(json.dumps({"generated_tokens": st.get("generated_tokens"), "error": st.get("error")}))
            return
        time.sleep(interval_ms / 1000.0)


# ------------------------------------------------------------------------------------------ ledger
def cmd_ledger(a):
    d = load_device()
    c = client(d)
    if a.action == "summary":
        print(json.dumps(c.ledger_summary(d["network_id"]), indent=2))
    else:
        ev = c.ledger_events(d["network_id"], limit=a.limit)
        if a.job_id:
            ev = [e for e in ev if e.get("job_id") == a.job_id]
        print(json.dumps(ev, indent=2))


# ------------------------------------------------------------------------------------------ pool
def _device_keypair():
    """This device's ed25519 key (from `mesh device init`); a fresh key if the device is not initialised."""
    from ..net import pki
    try:
        return pki.KeyPair.from_seed(bytes.fromhex(load_device()["private_key"]))
    except SystemExit:
        return pki.KeyPair()


def cmd_pool(a):
    """Pools (reference ``agent/src/pki``): a pool is an ed25519 root key; its id is derived from the
    root public key; members hold certificates signed by the root; `peers --listen-seconds` runs LAN
    beacon discovery for that long and records the verified peers."""
    from ..net import beacon, pki
    pools = home() / "pools"
    pools.mkdir(exist_ok=True)
    if a.action == "create":
        root = pki.KeyPair()
        dev = _device_keypair()
        cert = pki.MembershipCert.issue(dev.public, root, pki.ROLE_ADMIN)
        pid = root.pool_id.hex()
        (pools / f"{pid}.json").write_text(json.dumps({
            "pool_id": pid, "name": a.name, "root_public_key": root.public.hex(), "root_seed": root.seed().hex(),
            "role": "admin", "cert": cert.to_dict(), "created_at": int(time.time())}, indent=2))
        print(json.dumps({"pool_id": pid, "root_public_key": root.public.hex()}))
    elif a.action == "issue":
        p = json.loads((pools / f"{a.pool_id}.json").read_text())
        if "root_seed" not in p:
            raise SystemExit("only the pool admin (holder of the root key) can issue certificates")
        root = pki.KeyPair.from_seed(bytes.fromhex(p["root_seed"]))
        cert = pki.MembershipCert.issue(bytes.fromhex(a.device_pubkey), root,
                                        pki.ROLE_ADMIN if a.admin else pki.ROLE_MEMBER)
        print(json.dumps(cert.to_dict()))
    elif a.action == "join":
        entry = {"pool_id": a.pool_id, "name": a.name, "root_public_key": a.pool_root_pubkey, "role": "member",
                 "joined_at": int(time.time())}
        if pki.pool_id_from_pubkey(bytes.fromhex(a.pool_root_pubkey)).hex() != a.pool_id:
            raise SystemExit("pool id does not match the pool root public key")
        if a.cert:
            cert = pki.MembershipCert.from_dict(json.loads(Path(a.cert).read_text()))
            if not cert.verify(bytes.fromhex(a.pool_root_pubkey)):
                raise SystemExit("membership certificate does not verify against the pool root key")
            entry["cert"] = cert.to_dict()
            entry["role"] = cert.role
        (pools / f"{a.pool_id}.json").write_text(json.dumps(entry, indent=2))
        print(json.dumps({"pool_id": a.pool_id, "joined": True, "certified": "cert" in entry}))
    elif a.action == "list":
        out = []
        for f in sorted(pools.glob("*.json")):
            p = json.loads(f.read_text())
            p.pop("root_seed", None)
            out.append(p)
        print(json.dumps(out, indent=2))
    elif a.action == "peers":
        f = pools / f"{a.pool_id}.json"
        p = json.loads(f.read_text()) if f.exists() else {}
        if a.listen_seconds > 0 and "cert" in p:
            svc = beacon.BeaconService(_device_keypair(), [pki.MembershipCert.from_dict(p["cert"])],
                                       admin=p.get("role") == "admin").start()
            time.sleep(a.listen_seconds)
            peers = svc.peers(bytes.fromhex(a.pool_id))
            svc.close()
            p["peers"] = [{"node_id": x.node_id.hex(), "addr": f"{x.addr[0]}:{x.addr[1]}", "quic_port": x.quic_port,
                           "capabilities": x.capabilities, "last_seen": int(x.last_seen)} for x in peers]
            f.write_text(json.dumps(p, indent=2))
        print(json.dumps(p.get("peers", [])))
    else:
        print(json.dumps({"pools": len(list(pools.glob("*.json")))}))


# ------------------------------------------------------------------------------------------ model
def cmd_model(a):
    """The on-disk model store (``$MESHNET_MODEL_STORE``, default ``$MESHNET_HOME/models``) and the
    device's shard registry: import a Hugging Face Llama checkpoint, re-shard, list, describe."""
    from ..models.artifacts import model_store_dir
    from ..models.registry import ModelInfo, ShardRegistry
    store = Path(getattr(a, "store", None) or model_store_dir())
    if a.action == "import-hf":
        from ..models.convert import import_hf_llama
        out = import_hf_llama(a.src, store, a.model_id, a.workers)
        ShardRegistry(home() / "shards").register_model(ModelInfo.from_model_dir(out))
        print(json.dumps({"model_dir": str(out)}))
    elif a.action == "reshard":
        from ..models.convert import reshard
        out = reshard(store / a.model_id, Path(a.out) if a.out else store / f"{a.model_id}-tp{a.workers}", a.workers)
        print(json.dumps({"model_dir": str(out)}))
    elif a.action == "info":
        from dataclasses import asdict
        info = ModelInfo.from_model_dir(store / a.model_id, gpu_bytes=a.gpu_bytes or None)
        print(json.dumps(asdict(info), indent=2))
    else:
        models = sorted(p.parent.name for p in store.glob("*/model.json")) if store.exists() else []
        print(json.dumps({"store": str(store), "models": models,
                          "registry": ShardRegistry(home() / "shards").summary()}, indent=2))


# ------------------------------------------------------------------------------------------ doctor
def cmd_doctor(a):
    checks = []

    def check(name, fn):
        try:
            v = fn()
            checks.append({"check": name, "ok": True, "detail": v})
        except Exception as e:
            checks.append({"check": name, "ok": False, "detail": str(e)})

    import torch
    check("python", lambda: sys.version.split()[0])
    check("torch", lambda: torch.__version__)
    check("cuda_available", lambda: bool(torch.cuda.is_available()) or (_ for _ in ()).throw(
        RuntimeError("no CUDA device")))
    check("sm_100a", lambda: torch.cuda.get_device_capability(0) == (10, 0) or (_ for _ in ()).throw(
        RuntimeError(f"capability {torch.cuda.get_device_capability(0)}")))
    check("kernels_built", lambda: __import__("mesh_b200._C", fromlist=["x"]).__file__)
    check("runtime_built", lambda: __import__("mesh_b200._runtime", fromlist=["x"]).__file__)
    check("nccl", lambda: ".".join(map(str, torch.cuda.nccl.version())))
    if a.stage == "production":
        check("device_config", lambda: load_device()["device_id"])
        check("control_plane", lambda: client(load_device()).health())
    print(json.dumps(checks, indent=2))
    return 0 if all(c["ok"] for c in checks) else 1


# ------------------------------------------------------------------------------------------ ui
def cmd_ui(a):
    """Local API for dashboards (``/api/local/*``, the routes of ``agent/src/ui.rs:583-612``); the
    browser dashboard itself is not shipped."""
    import uvicorn
    from .local_api import create_local_app
    uvicorn.run(create_local_app(), host="127.0.0.1", port=a.api_port)


def build_parser():
    p = argparse.ArgumentParser(prog="mesh", description="mesh_b200 CLI")
    sub = p.add_subparsers(dest="cmd", required=True)
    dev = sub.add_parser("device").add_subparsers(dest="action", required=True)
    i = dev.add_parser("init")
    i.add_argument("-n", "--network-id", required=True)
    i.add_argument("-d", "--name", default="My Device")
    i.add_argument("-c", "--control-plane", default="http://localhost:8080")
    i.add_argument("--preferred-provider", choices=["cpu", "cuda"])
    i.add_argument("--device-id")
    i.add_argument("--tp", type=int, default=1, help="GPUs of this box that serve as one tensor-parallel group")
    i.add_argument("--model-dir", default="", help="on-disk model (model.json + shards) the group loads")
    i.set_defaults(fn=cmd_device_init)
    s = dev.add_parser("start")
    s.add_argument("-l", "--log-level", default="info")
    s.add_argument("--no-restart", action="store_true")
    s.set_defaults(fn=cmd_device_start)
    r = dev.add_parser("runtime")
    r.add_argument("-l", "--log-level", default="info")
    r.set_defaults(fn=cmd_device_runtime)
    dev.add_parser("status").set_defaults(fn=cmd_device_status)
    res = sub.add_parser("resource").add_subparsers(dest="action", required=True)
    lk = res.add_parser("lock")
    lk.add_argument("-m", "--memory", required=True)
    lk.set_defaults(fn=cmd_resource)
    res.add_parser("unlock").set_defaults(fn=cmd_resource)
    res.add_parser("status").set_defaults(fn=cmd_resource)
    ring = sub.add_parser("ring").add_subparsers(dest="action", required=True)
    j = ring.add_parser("join")
    j.add_argument("-m", "--model-id", required=True)
    j.add_argument("-M", "--memory")
    j.set_defaults(fn=cmd_ring)
    for n in ("leave", "status", "topology", "shard"):
        ring.add_parser(n).set_defaults(fn=cmd_ring)
    job = sub.add_parser("job").add_subparsers(dest="action", required=True)
    jr = job.add_parser("run")
    jr.add_argument("-p", "--prompt", required=True)
    jr.add_argument("-m", "--model-id", default="tinyllama-1.1b")
    jr.add_argument("-n", "--max-tokens", type=int, default=100)
    jr.add_argument("-t", "--temperature", type=float, default=1.0)
    jr.add_argument("--top-p", type=float, default=0.9)
    jr.add_argument("--wait", action="store_true")
    jr.set_defaults(fn=cmd_job)
    js = job.add_parser("status")
    js.add_argument("--job-id", required=True)
    js.set_defaults(fn=cmd_job)
    jw = job.add_parser("watch")
    jw.add_argument("--job-id", required=True)
    jw.add_argument("--interval-ms", type=int, default=2000)
    jw.set_defaults(fn=cmd_job)
    job.add_parser("stats").set_defaults(fn=cmd_job)
    led = sub.add_parser("ledger").add_subparsers(dest="action", required=True)
    ls = led.add_parser("summary")
    ls.add_argument("--job-id")
    ls.set_defaults(fn=cmd_ledger)
    le = led.add_parser("events")
    le.add_argument("--job-id")
    le.add_argument("--limit", type=int, default=20)
    le.set_defaults(fn=cmd_ledger)
    pool = sub.add_parser("pool").add_subparsers(dest="action", required=True)
    pc = pool.add_parser("create")
    pc.add_argument("-n", "--name", required=True)
    pc.set_defaults(fn=cmd_pool)
    pj = pool.add_parser("join")
    pj.add_argument("--pool-id", required=True)
    pj.add_argument("--pool-root-pubkey", required=True)
    pj.add_argument("-n", "--name")
    pj.add_argument("--cert", help="membership certificate (JSON) issued by the pool admin")
    pj.set_defaults(fn=cmd_pool)
    pool.add_parser("list").set_defaults(fn=cmd_pool)
    pp = pool.add_parser("peers")
    pp.add_argument("--pool-id", required=True)
    pp.add_argument("--listen-seconds", type=float, default=0.0, help="run LAN beacon discovery this long")
    pi = pool.add_parser("issue")
    pi.add_argument("--pool-id", required=True)
    pi.add_argument("--device-pubkey", required=True)
    pi.add_argument("--admin", action="store_true")
    pi.set_defaults(fn=cmd_pool)
    pp.set_defaults(fn=cmd_pool)
    pool.add_parser("status").set_defaults(fn=cmd_pool)
    mdl = sub.add_parser("model").add_subparsers(dest="action", required=True)
    mi = mdl.add_parser("import-hf", help="import a local Hugging Face Llama checkpoint into the model store")
    mi.add_argument("--src", required=True)
    mi.add_argument("--model-id", required=True)
    mi.add_argument("--workers", type=int, default=1)
    mi.add_argument("--store")
    mr = mdl.add_parser("reshard", help="rewrite an on-disk model for another worker count")
    mr.add_argument("--model-id", required=True)
    mr.add_argument("--workers", type=int, required=True)
    mr.add_argument("--store")
    mr.add_argument("--out")
    mdl.add_parser("list", help="models in the store and shards in this device's registry").set_defaults(fn=cmd_model)
    ms = mdl.add_parser("info", help="one model's description (memory per worker, valid TP degrees)")
    ms.add_argument("--model-id", required=True)
    ms.add_argument("--store")
    ms.add_argument("--gpu-bytes", type=int, default=0)
    for q in (mi, mr, ms):
        q.set_defaults(fn=cmd_model)
    doc = sub.add_parser("doctor")
    doc.add_argument("--stage", choices=["preflight", "production"], default="production")
    doc.set_defaults(fn=cmd_doctor)
    ui = sub.add_parser("ui")
    ui.add_argument("--port", type=int, default=43110)
    ui.add_argument("--api-port", type=int, default=43111)
    ui.add_argument("--api-only", action="store_true")
    ui.set_defaults(fn=cmd_ui)
    return p


def main(argv=None):
    a = build_parser().parse_args(argv)
    rc = a.fn(a)
    return rc if isinstance(rc, int) else 0


if __name__ == "__main__":
    sys.exit(main())
