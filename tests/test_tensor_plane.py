"""TCP tensor plane (reference frame format) and CPU ring all-reduce / TP forward on loopback."""
import threading

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
