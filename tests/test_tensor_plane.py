"""TCP tensor plane (reference frame format) and CPU ring all-reduce / TP forward on loopback."""
import threading
import time

import numpy as np
import pytest
from hypothesis import given, settings, strategies as st

from mesh_b200.config import get_preset
from mesh_b200.models.sharding import shard_layout
from mesh_b200.models.weights import synthetic_reference_weights
from mesh_b200.oracle.forward import LocalForwardPass
from mesh_b200.oracle.tp_forward import ShardedForwardPass, shard_reference_weights
from mesh_b200.parallel.tcp_plane import TensorPlane, TensorPlaneError, WorkerRing


def _rings(n, **kw):
    planes = [TensorPlane() for _ in range(n)]
    addrs = [p.addr for p in planes]
    return planes, [WorkerRing(planes[i], i, addrs, **kw) for i in range(n)]


def _par(fns):
    out, err = [None] * len(fns), []

    def run(i):
        try:
            out[i] = fns[i]()
        except Exception as e:  # pragma: no cover
            err.append(e)
    th = [threading.Thread(target=run, args=(i,)) for i in range(len(fns))]
    [t.start() for t in th]
    [t.join(60) for t in th]
    assert not err, err
    return out


@pytest.mark.parametrize("n", [2, 3, 5])
def test_ring_allreduce_sum_identical_on_all_ranks(n):
    planes, rings = _rings(n)
    rng = np.random.default_rng(n)
    xs = [rng.standard_normal((7, 33)).astype(np.float32) for _ in range(n)]
    outs = _par([lambda i=i: rings[i].all_reduce(xs[i], layer=3) for i in range(n)])
    want = sum(xs)
    for o in outs:
        np.testing.assert_allclose(o, want, rtol=1e-5, atol=1e-5)
    assert all(np.array_equal(outs[0], o) for o in outs)  # identical across ranks
    _par([lambda i=i: rings[i].barrier() for i in range(n)])
    for p in planes:
        p.close()


@settings(max_examples=10, deadline=None)
@given(st.integers(1, 300), st.integers(2, 4))
def test_ring_allreduce_any_length(length, n):
    planes, rings = _rings(n)
    xs = [np.full(length, float(i + 1), np.float32) for i in range(n)]
    outs = _par([lambda i=i: rings[i].all_reduce(xs[i]) for i in range(n)])
    for o in outs:
        np.testing.assert_allclose(o, np.full(length, n * (n + 1) / 2))
    for p in planes:
        p.close()


def test_receive_timeout_and_oversized_rejection():
    p = TensorPlane(max_message_bytes=1024)
    with pytest.raises(TimeoutError):
        p.recv(collective_id=b"\0" * 16, seq=1, sender=0, timeout_s=0.2)
    with pytest.raises(TensorPlaneError):
        p.send(p.addr, np.zeros(1000, np.float32), collective_id=b"\0" * 16, seq=1, sender=0)
    p.close()


def test_tp2_cpu_forward_over_loopback_matches_oracle():
    cfg = get_preset("tiny")
    w = synthetic_reference_weights(cfg, seed=13)
    planes, rings = _rings(2)
    fps = [ShardedForwardPass(cfg, shard_layout(cfg, r, 2), shard_reference_weights(w, shard_layout(cfg, r, 2)),
                              rings[r]) for r in range(2)]
    prompt = [4, 8, 15, 16, 23, 42]
    outs = _par([lambda r=r: fps[r].generate(prompt, 6) for r in range(2)])
    want = LocalForwardPass(w).generate(prompt, 6)
    assert outs[0] == outs[1] == want
    assert fps[0].allreduce_calls == 2 * cfg.num_layers * 6  # two per layer per forward
    assert planes[0].metrics.bytes_sent > 0
    for p in planes:
        p.close()


# ------------------------------------------------------------------------------ flow control
from mesh_b200.parallel.tcp_plane import (HEADER, PlaneConfig, TokenBucket,  # noqa: E402
                                          lane_stream_count)

CID = b"\x07" * 16
MiB = 1024 * 1024


def test_budget_split_and_lane_stream_policy():
    c = PlaneConfig(max_message_bytes=MiB, max_outbound_inflight_bytes=64 * MiB).sanitized()
    assert c.priority_budget == 16 * MiB and c.bulk_budget == 48 * MiB and c.per_peer_bulk_budget == 24 * MiB
    small = PlaneConfig(max_message_bytes=MiB, max_outbound_inflight_bytes=2 * MiB).sanitized()
    assert small.priority_budget == MiB + HEADER  # at least one whole frame
    assert small.bulk_budget == MiB + HEADER and small.per_peer_bulk_budget == MiB + HEADER
    # control is one stream everywhere; cpu ranks and fit-first jobs one stream per lane
    for lane in ("reduce_scatter", "all_gather", "control", "bulk_transfer", "checkpoint"):
        assert lane_stream_count(lane, "lan", "cpu", "throughput_first", 3) == 1
        assert lane_stream_count(lane, "lan", "cuda", "fit_first", 3) == 1
    assert lane_stream_count("control", "lan", "cuda", "throughput_first", 3) == 1
    assert lane_stream_count("reduce_scatter", "lan", "cuda", "throughput_first", 3) == 3
    assert lane_stream_count("all_gather", "lan", "cuda", "throughput_first", 3) == 2
    assert lane_stream_count("reduce_scatter", "conservative", "cuda", "throughput_first", 4) == 2
    assert lane_stream_count("checkpoint", "lan", "cuda", "latency_first", 3) == 1
    with pytest.raises(ValueError):
        PlaneConfig(profile="wan").sanitized()


def test_multi_stream_lane_pools_connections_and_keeps_order_per_slot():
    rx = TensorPlane()
    tx = TensorPlane(config=PlaneConfig(provider="cuda", max_streams_per_peer=3))
    assert tx.stream_count("reduce_scatter") == 3 and tx.stream_count("control") == 1
    for stream in range(6):
        for k in range(3):
            tx.send(rx.addr, np.full(5, 10 * stream + k, np.float32), collective_id=CID, seq=1, sender=0,
                    stream=stream, lane="reduce_scatter")
    tx.send(rx.addr, np.ones(2, np.float32), collective_id=CID, seq=1, sender=0, lane="control")
    for stream in range(6):
        for k in range(3):  # frames of one slot arrive in send order
            got = rx.recv(collective_id=CID, seq=1, sender=0, stream=stream, lane="reduce_scatter", timeout_s=5)
            assert got[0] == 10 * stream + k
    rx.recv(collective_id=CID, seq=1, sender=0, lane="control", timeout_s=5)
    m = tx.metrics_snapshot()
    assert m["current_outbound_connections"] == 4  # 3 reduce-scatter streams + 1 control
    assert m["per_class_sends"] == {"bulk": 18, "latency_critical": 1}
    assert rx.metrics_snapshot()["current_inbound_queued_bytes"] == 0
    tx.close()
    rx.close()


def test_bulk_backlog_does_not_block_priority_frames():
    """With the bulk budget exhausted (e.g. a checkpoint upload in flight), a control frame still
    goes out at once while another bulk frame waits and then times out, counted."""
    rx = TensorPlane()
    tx = TensorPlane(config=PlaneConfig(max_message_bytes=64 * 1024, max_outbound_inflight_bytes=1 * MiB,
                                        io_timeout_s=0.3))
    tx._out_bulk.acquire(tx._out_bulk.capacity, 1.0)  # the backlog
    t0 = time.monotonic()
    tx.send(rx.addr, np.ones(16, np.float32), collective_id=CID, seq=2, sender=0, lane="control")
    tx.send(rx.addr, np.ones(16, np.float32), collective_id=CID, seq=2, sender=0, lane="all_gather")
    assert time.monotonic() - t0 < 0.25
    with pytest.raises(TensorPlaneError):
        tx.send(rx.addr, np.ones(16, np.float32), collective_id=CID, seq=2, sender=0, lane="checkpoint")
    m = tx.metrics_snapshot()
    assert m["send_timeouts"] == 1 and m["per_class_sends"] == {"latency_critical": 1, "interactive": 1}
    tx._out_bulk.release(tx._out_bulk.capacity)
    tx.send(rx.addr, np.ones(16, np.float32), collective_id=CID, seq=2, sender=0, lane="checkpoint")
    assert rx.recv(collective_id=CID, seq=2, sender=0, lane="checkpoint", timeout_s=5).sum() == 16
    tx.close()
    rx.close()


def test_per_peer_bulk_budget_isolates_peers():
    a, b = TensorPlane(), TensorPlane()
    tx = TensorPlane(config=PlaneConfig(max_message_bytes=64 * 1024, max_outbound_inflight_bytes=1 * MiB,
                                        io_timeout_s=0.3))
    peer_a = tx._budgets(tuple(a.addr), "bulk")[2]
    peer_a.acquire(peer_a.capacity, 1.0)  # peer A's share is taken
    tx.send(b.addr, np.ones(8, np.float32), collective_id=CID, seq=3, sender=0, lane="bulk_transfer")
    with pytest.raises(TensorPlaneError):
        tx.send(a.addr, np.ones(8, np.float32), collective_id=CID, seq=3, sender=0, lane="bulk_transfer")
    peer_a.release(peer_a.capacity)
    assert b.recv(collective_id=CID, seq=3, sender=0, lane="bulk_transfer", timeout_s=5).sum() == 8
    for p in (a, b, tx):
        p.close()


def test_inbound_budget_pushes_back_without_loss():
    """A receiver whose mailbox holds its message budget stops reading; the frames behind wait in
    TCP and are admitted, in order, as the consumer takes frames out."""
    rx = TensorPlane(config=PlaneConfig(max_inbound_messages=2, io_timeout_s=10))
    tx = TensorPlane()
    for k in range(5):
        tx.send(rx.addr, np.full(4, k, np.float32), collective_id=CID, seq=4, sender=1, lane="all_gather")
    time.sleep(0.3)
    m = rx.metrics_snapshot()
    assert m["receive_count"] == 2 and m["inbound_backpressure_waits"] >= 1
    got = [rx.recv(collective_id=CID, seq=4, sender=1, lane="all_gather", timeout_s=5)[0] for _ in range(5)]
    assert got == [0, 1, 2, 3, 4]
    assert rx.metrics_snapshot()["inbound_queue_full_rejections"] == 0
    tx.close()
    rx.close()


def test_inbound_budget_drops_when_nobody_reads():
    rx = TensorPlane(config=PlaneConfig(max_inbound_messages=1, io_timeout_s=0.2))
    tx = TensorPlane()
    for k in range(3):
        tx.send(rx.addr, np.full(4, k, np.float32), collective_id=CID, seq=5, sender=1, lane="all_gather")
    time.sleep(0.8)
    assert rx.metrics_snapshot()["inbound_queue_full_rejections"] >= 1
    assert rx.recv(collective_id=CID, seq=5, sender=1, lane="all_gather", timeout_s=1)[0] == 0
    tx.close()
    rx.close()


def test_send_refreshes_a_broken_connection_once():
    rx = TensorPlane()
    tx = TensorPlane()
    tx.send(rx.addr, np.ones(3, np.float32), collective_id=CID, seq=6, sender=0, lane="control")
    rx.recv(collective_id=CID, seq=6, sender=0, lane="control", timeout_s=5)
    for pool in tx._pools.values():  # break the pooled socket under the plane
        for c in pool:
            c.sock.close()
    tx.send(rx.addr, np.full(3, 2.0, np.float32), collective_id=CID, seq=7, sender=0, lane="control")
    assert rx.recv(collective_id=CID, seq=7, sender=0, lane="control", timeout_s=5).sum() == 6
    m = tx.metrics_snapshot()
    assert m["connection_refresh_attempts"] == 1 and m["connection_refresh_successes"] == 1
    assert m["connection_evictions"] == 1
    tx.close()
    rx.close()
    dead = TensorPlane(config=PlaneConfig(connect_timeout_s=0.5))
    with pytest.raises(TensorPlaneError):
        dead.send(rx.addr, np.ones(1, np.float32), collective_id=CID, seq=8, sender=0)
    dead.close()


@pytest.mark.parametrize("n", [0, 1, 5, 4099])
def test_raw_bytes_frames_and_background_send(n):
    rx, tx = TensorPlane(), TensorPlane()
    payload = bytes((i * 7) % 251 for i in range(n))
    fut = tx.spawn(rx.addr, payload, collective_id=CID, seq=9, sender=2, slot=n, lane="checkpoint")
    fut.result(timeout=10)
    assert rx.recv_bytes(collective_id=CID, seq=9, sender=2, slot=n, lane="checkpoint", timeout_s=5) == payload
    assert tx.metrics_snapshot()["per_lane_sent"] == {"checkpoint": 4 * ((4 + n + 3) // 4)}
    tx.close()
    rx.close()


def test_bulk_pacing_token_bucket():
    tb = TokenBucket(200_000)
    assert tb.take(200_000) == 0.0  # one second of burst credit
    t0 = time.monotonic()
    w = tb.take(100_000)
    assert 0.4 < w < 0.6 and time.monotonic() - t0 >= 0.4
    assert TokenBucket(0).take(10 ** 9) == 0.0
