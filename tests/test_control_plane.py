"""Control plane on CPU: policies, ring topology, job lifecycle over HTTP with a worker, failover."""
import socket
import threading
import time

import pytest

from mesh_b200.config import get_preset
from mesh_b200.control_plane import policy
from mesh_b200.control_plane.db import Database
from mesh_b200.control_plane.service import ControlPlane, Conflict
from mesh_b200.engine.backend import CpuReferenceBackend
from mesh_b200.engine.coordinator import InferenceCoordinator
from mesh_b200.models.weights import synthetic_reference_weights
from mesh_b200.oracle.forward import LocalForwardPass


def test_consumption_quote_reference_example():
    # control-plane/src/consumption_policy.rs tests: 8 prompt + 4 completion on a 64 GiB model
    q = policy.consumption(8, 4, 64 * 1024 ** 3)
    assert q["model_size_factor"] == 2.0 and q["total_credits"] == 24.0
    assert policy.consumption(8, 4, 1024 ** 3)["model_size_factor"] == 1.0


def test_credit_policy_shares_sum_to_budget_and_clamp():
    a = [policy.AssignmentCreditInput("a", 1000, 4, 0, 1024, 0),
         policy.AssignmentCreditInput("b", 10, 4, 1024, 2048, 0)]  # b is 100x faster -> clamped 1.5
    out = policy.credit_policy(10, 10, 32 * 1024 ** 3, 2048, a)
    assert abs(sum(x["credits"] for x in out["assignments"]) - out["job_credit_budget"]) < 1e-9
    tm = {x["device_id"]: x["throughput_multiplier"] for x in out["assignments"]}
    assert tm["b"] == 1.5 and tm["a"] == 0.5


def test_weighted_group_ranges():
    r = policy.weighted_group_ranges(4096, 512, [1, 1])
    assert r == [(0, 2048), (2048, 4096)]
    r = policy.weighted_group_ranges(4096, 512, [3, 1])
    assert r[0][1] % 512 == 0 and r[0][1] > 2048 and r[-1][1] == 4096
    with pytest.raises(ValueError):
        policy.weighted_group_ranges(4096, 3000, [1])


def _cp():
    return ControlPlane(Database())


def test_ring_join_leave_topology():
    cp = _cp()
    net = cp.create_network("n")["network_id"]
    for d, mem in (("d0", 8 << 30), ("d1", 8 << 30)):
        cp.register_device(d, net, tier="tier2", contributed_memory=mem)
    t = cp.join_ring("d0", net, "llama3-8b", 8 << 30)
    assert t["stable"] and t["workers"][0]["column_end"] == 4096
    t = cp.join_ring("d1", net, "llama3-8b", 8 << 30)
    w = t["workers"]
    assert [x["column_start"] for x in w] == [0, 2048] and w[0]["right_neighbor"] == "d1"
    assert all(x["column_start"] % 512 == 0 for x in w)  # GQA group width 4*128
    v = t["version"]
    t = cp.leave_ring("d1")
    assert t["version"] == v + 1 and t["workers"][0]["column_end"] == 4096


def test_submit_requires_stable_ring():
    cp = _cp()
    net = cp.create_network("n")["network_id"]
    with pytest.raises(Conflict):
        cp.submit_inference(net, "tiny", prompt_tokens=[1, 2])


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.fixture
def server():
    import uvicorn
    from mesh_b200.control_plane.app import create_app
    cp = _cp()
    app = create_app(cp, presence_interval_s=0)
    port = _free_port()
    cfg = uvicorn.Config(app, host="127.0.0.1", port=port, log_level="error")
    srv = uvicorn.Server(cfg)
    th = threading.Thread(target=srv.run, daemon=True)
    th.start()
    for _ in range(100):
        if srv.started:
            break
        time.sleep(0.05)
    yield cp, f"http://127.0.0.1:{port}"
    srv.should_exit = True
    th.join(timeout=5)


def test_job_lifecycle_over_http_with_worker(server):
    from mesh_b200.runtime.client import ControlPlaneClient
    from mesh_b200.runtime.worker import Worker
    cp, url = server
    c = ControlPlaneClient(url)
    assert c.health()["status"] == "ok"
    net = c.create_network("lan")["network_id"]
    weights = synthetic_reference_weights(get_preset("tiny"), seed=5)
    coord = InferenceCoordinator(CpuReferenceBackend(weights))
    w = Worker(c, "gpu0", net, "tiny", coord, heartbeat_interval_s=0.2)
    w.start()
    c.register(device_id="client", network_id=net)
    jobs = [c.submit(net, "tiny", prompt_tokens=p, max_tokens=5, temperature=0.0, submitter_device_id="client")
            for p in ([1, 2, 3], [7, 7, 7, 7])]
    assert all(j["status"] == "pending" for j in jobs)
    kinds = [w.run_once() for _ in range(4)]
    assert kinds.count("prefill") == 2 and "decode" in kinds
    for j, p in zip(jobs, ([1, 2, 3], [7, 7, 7, 7])):
        st = c.job(j["job_id"])
        assert st["status"] == "completed", st
        assert st["generated_tokens"] == LocalForwardPass(weights).generate(p, 5)
    summary = c.ledger_summary(net)
    assert summary["earned"]["gpu0"] > 0 and abs(summary["outstanding_reserved"]) < 1e-6
    st = c.scheduler_status(net)
    assert st["peak_batch_size"] >= 2 and st["jobs"]["completed"] == 2
    w.stop()


def test_failover_prefill_loss_fails_and_decode_loss_regroups():
    cp = _cp()
    net = cp.create_network("n")["network_id"]
    for d in ("a", "b", "c"):
        cp.register_device(d, net)
    cp.join_ring("a", net, "tiny")
    cp.join_ring("b", net, "tiny")
    j1 = cp.submit_inference(net, "tiny", prompt_tokens=[1, 2], max_tokens=4, submitter_device_id="a")
    j2 = cp.submit_inference(net, "tiny", prompt_tokens=[3, 4], max_tokens=4, submitter_device_id="a")
    # job 2 finished prefill on both ranks and has a checkpoint
    for d in ("a", "b"):
        cp.claim(d)
        cp.claim(d)
        cp.report_progress(j2["job_id"], d, "prefill", 1, kv_cache_seq_len=2)
    cp.upload_session_checkpoint(j2["job_id"], j2["session_id"], b"ckpt", source_device_id="a")
    cp.join_ring("c", net, "tiny")
    # c serves a full replica of the model (as after a shard handoff): it can replace b
    with cp.db.tx() as c:
        c.execute("UPDATE ring_members SET column_start=0, column_end=512 WHERE device_id='c'")
    decisions = {d["job_id"]: d for d in cp.evaluate_failover(["b"])}
    assert decisions[j1["job_id"]]["strategy"] == "fail"
    assert cp.job_status(j1["job_id"])["status"] == "failed"
    d2 = decisions[j2["job_id"]]
    assert d2["strategy"] == "replace" and d2["resume_mode"] == "requires_checkpoint_transfer"
    assert d2["recovery_state"] == "paused" and d2["participant_device_ids"] == ["c"]
    assert d2["transfer_source_device_id"] == "a"
    st = cp.job_status(j2["job_id"])
    assert st["decode_queue"]["status"] == "blocked_on_transfer"
    assert [m["device_id"] for m in st["plan"]["execution_groups"][1]["members"]] == ["c"]
    # the replacement is not claimable until the KV arrives; the transfer completes -> ready
    assert cp.claim("c")["kind"] == "idle"
    t = cp.pending_kv_transfers("c")
    assert len(t) == 1 and t[0]["source_device_id"] == "a"
    cp.report_kv_transfer(j2["job_id"], j2["session_id"], "a", "c", status="completed",
                          transfer_id=t[0]["transfer_id"])
    assert cp.job_status(j2["job_id"])["decode_queue"]["status"] == "ready"
    w = cp.claim("c")
    assert w["kind"] == "decode" and w["assignments"][0]["session_id"] == j2["session_id"]
    ev = cp.ledger_summary(net)
    assert ev["events"] > 0


def test_failover_shrinks_to_a_surviving_full_replica_and_cleans_up():
    cp = _cp()
    net = cp.create_network("n")["network_id"]
    for d in ("a", "b"):
        cp.register_device(d, net)
    cp.join_ring("a", net, "tiny")
    cp.join_ring("b", net, "tiny")
    j = cp.submit_inference(net, "tiny", prompt_tokens=[5, 6], max_tokens=4, submitter_device_id="a")
    for d in ("a", "b"):
        cp.claim(d)
        cp.report_progress(j["job_id"], d, "prefill", 1, kv_cache_seq_len=2)
    assert cp.claim("a")["kind"] == "decode"
    # b is lost while a, which also holds every column of the decode group, keeps serving
    with cp.db.tx() as c:
        c.execute("UPDATE ring_members SET column_start=0, column_end=512 WHERE device_id='a'")
    plan = cp.job_status(j["job_id"])["plan"]
    for m in plan["execution_groups"][1]["members"]:
        m["shard_column_start"], m["shard_column_end"] = 0, 512
    with cp.db.tx() as c:
        c.execute("UPDATE inference_jobs SET plan=? WHERE job_id=?", (__import__("json").dumps(plan), j["job_id"]))
    d = cp.evaluate_failover(["b"])[0]
    assert d["strategy"] == "shrink" and d["resume_mode"] == "immediate" and d["participant_device_ids"] == ["a"]
    assert cp.job_status(j["job_id"])["decode_queue"]["status"] == "ready"
    # a finished job keeps no leases after cleanup
    cp.cancel_job(j["job_id"])
    with cp.db.tx() as c:
        c.execute("UPDATE inference_decode_queue SET lease_id='stale' WHERE job_id=?", (j["job_id"],))
    out = cp.cleanup_terminal_state()
    assert out["queue_leases_released"] == 1
    assert cp.job_status(j["job_id"])["decode_queue"]["lease_id"] is None


def test_claim_reports_blocked_reasons_and_respects_group_leader():
    cp = _cp()
    net = cp.create_network("n")["network_id"]
    for d in ("a", "b"):
        cp.register_device(d, net)
    cp.join_ring("a", net, "tiny")
    cp.join_ring("b", net, "tiny")
    cp.submit_inference(net, "tiny", prompt_tokens=[1, 2], max_tokens=4)
    # the follower cannot open the prefill group; the leader can, then the follower joins it
    w = cp.claim("b")
    assert w["kind"] == "idle" and w["blocked"][0]["reason"] == "lease_held_by_peer"
    assert cp.claim("a")["kind"] == "prefill"
    assert cp.claim("b")["kind"] == "prefill"
    ev = cp.db.query("SELECT * FROM inference_scheduler_events WHERE event='claim_blocked'")
    assert ev and "lease_held_by_peer" in ev[0]["details"]


def test_disaggregated_plan_blocks_decode_until_checkpoint_arrives():
    cp = _cp()
    net = cp.create_network("n")["network_id"]
    for d, tier in (("a", "tier2"), ("b", "tier2"), ("c", "tier3")):
        cp.register_device(d, net, tier=tier)
    for d in ("a", "b", "c"):
        cp.join_ring(d, net, "tiny")
    # a and b tile the columns (the prefill TP group); c, a larger worker, holds a full replica and
    # scores best for decode, so the plan hands the KV from the prefill group to c by checkpoint
    with cp.db.tx() as c:
        c.execute("UPDATE ring_members SET column_start=0, column_end=256 WHERE device_id='a'")
        c.execute("UPDATE ring_members SET column_start=256, column_end=512 WHERE device_id='b'")
        c.execute("UPDATE ring_members SET column_start=0, column_end=512 WHERE device_id='c'")
    j = cp.submit_inference(net, "tiny", prompt_tokens=[1, 2, 3], max_tokens=3)
    plan = j["plan"]
    assert plan["kv_transfer_policy"] == "checkpoint_handoff"
    assert [m["device_id"] for m in plan["execution_groups"][0]["members"]] == ["a", "b"]
    assert [m["device_id"] for m in plan["execution_groups"][1]["members"]] == ["c"]
    for d in ("a", "b"):
        assert cp.claim(d)["kind"] == "prefill"
        cp.report_progress(j["job_id"], d, "prefill", 1, kv_cache_seq_len=3)
    assert cp.job_status(j["job_id"])["decode_queue"]["status"] == "blocked_on_transfer"
    cp.upload_session_checkpoint(j["job_id"], j["session_id"], b"kv", source_device_id="a")
    assert cp.job_status(j["job_id"])["decode_queue"]["status"] == "ready"
    assert cp.claim("c")["kind"] == "decode"


def test_presence_marks_stale_and_reconciles_leases():
    cp = _cp()
    cp.stale_timeout_s = 0.5
    net = cp.create_network("n")["network_id"]
    cp.register_device("a", net)
    cp.join_ring("a", net, "tiny")
    assert cp.presence_sweep(now=time.time()) == []
    assert cp.presence_sweep(now=time.time() + 1.0) == ["a"]
    assert not cp.topology(net, "tiny")["stable"]
    cp.heartbeat("a")
    assert cp.topology(net, "tiny")["stable"]
    j = cp.submit_inference(net, "tiny", prompt_tokens=[1], max_tokens=2)
    w = cp.claim("a")
    assert w["kind"] == "prefill"
    # an expired lease goes back to pending
    with cp.db.tx() as c:
        c.execute("UPDATE inference_job_assignments SET lease_expires=0 WHERE job_id=?", (j["job_id"],))
    assert cp.reconcile_stale_leases() == 1
    assert cp.claim("a")["kind"] == "prefill"
