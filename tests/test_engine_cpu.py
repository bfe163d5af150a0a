"""Engine semantics on CPU: native scheduler, coordinator over the oracle backend, checkpoints."""
import os
import random

import numpy as np
import pytest
from hypothesis import given, settings, strategies as st

from mesh_b200 import _runtime
from mesh_b200.config import EngineConfig, get_preset
from mesh_b200.engine.backend import CpuReferenceBackend, token_ceiling
from mesh_b200.engine.checkpoint import Checkpoint, CheckpointConfig, CheckpointManager
from mesh_b200.engine.coordinator import InferenceCoordinator, RecoveryGovernor, _PyDecodeScheduler
from mesh_b200.engine.stats import InferenceStats
from mesh_b200.engine.types import (ExecutionPhase, GenerationConfig, InferenceRequest, PrefillComplete,
                                    SessionPauseReason, SessionRuntimeStatus)
from mesh_b200.models.weights import synthetic_reference_weights
from mesh_b200.oracle.forward import LocalForwardPass


# ------------------------------------------------------------------------------------ scheduler
def test_page_allocator_native():
    a = _runtime.PageAllocator(8, 1)
    p = a.alloc(3)
    assert p == [1, 2, 3] and a.num_free == 4
    assert a.alloc(5) is None
    a.free([2])
    assert a.alloc(1) == [2]
    with pytest.raises(ValueError):
        a.free([7])


def _fill(s, kvs, mode=1, cls=None, ceil=None):
    for i, kv in enumerate(kvs):
        s.register_session(i, 0 if cls is None else cls[i], kv, -1 if ceil is None else ceil[i], mode)
        s.enqueue(i)


def test_fair_order_by_steps_served_then_epoch():
    s = _runtime.DecodeScheduler()
    _fill(s, [100, 100, 100])
    b = s.build_batch(-1, 2, 10 ** 9)
    assert [x[0] for x in b["slots"]] == [0, 1]
    assert b["deferred_for_capacity"] == 1
    for sid in (0, 1):
        s.served(sid)
        s.enqueue(sid)
    # session 2 has served fewer steps: it goes first now
    b = s.build_batch(-1, 2, 10 ** 9)
    assert [x[0] for x in b["slots"]][0] == 2


def test_skew_guardrail_throughput_vs_latency_vs_fit():
    for mode, admitted in ((1, {0, 1}), (2, {0, 1}), (0, {0, 1, 2})):
        s = _runtime.DecodeScheduler()
        _fill(s, [1000, 1400, 3000], mode=mode)
        b = s.build_batch(-1, 8, 10 ** 9)
        assert {x[0] for x in b["slots"]} == admitted, mode
    s = _runtime.DecodeScheduler()
    _fill(s, [1000, 1600], mode=2)  # latency: max <= max(1.5*min, min+256) = 1500
    assert len(s.build_batch(-1, 8, 10 ** 9)["slots"]) == 1


def test_kv_budget_and_primary_and_class_cohesion():
    s = _runtime.DecodeScheduler()
    _fill(s, [500, 500, 500], cls=[0, 1, 0])
    b = s.build_batch(2, 8, 900)
    assert b["slots"][0][0] == 2                 # primary first
    assert b["deferred_for_guardrail"] == 1      # class 1 deferred
    assert b["deferred_for_kv_budget"] == 1      # 500 + 500 > 900
    s2 = _runtime.DecodeScheduler()
    _fill(s2, [100, 100], ceil=[2048, 8192])
    assert len(s2.build_batch(-1, 8, 10 ** 9)["slots"]) == 1  # fast-path bucket cohesion


@settings(max_examples=60, deadline=None)
@given(st.lists(st.tuples(st.integers(1, 5000), st.integers(0, 2), st.sampled_from([-1, 2048, 8192])),
                min_size=1, max_size=12),
       st.integers(0, 3), st.integers(1, 6), st.integers(100, 20000), st.integers(-1, 11))
def test_native_scheduler_equals_python_restatement(sess, mode, max_batch, max_kv, primary):
    a, b = _runtime.DecodeScheduler(), _PyDecodeScheduler()
    for i, (kv, c, ce) in enumerate(sess):
        for s in (a, b):
            s.register_session(i, c, kv, ce, mode)
            s.enqueue(i)
    for _ in range(3):
        ra = a.build_batch(primary, max_batch, max_kv)
        rb = b.build_batch(primary, max_batch, max_kv)
        assert [tuple(x) for x in ra["slots"]] == [tuple(x) for x in rb["slots"]]
        assert ra["deferred_for_capacity"] == rb["deferred_for_capacity"]
        assert ra["deferred_for_guardrail"] == rb["deferred_for_guardrail"]
        assert ra["deferred_for_kv_budget"] == rb["deferred_for_kv_budget"]
        for sid, *_ in ra["slots"]:
            for s in (a, b):
                s.served(sid)
                s.enqueue(sid)
        assert a.queued() == b.queued()


def test_frame_header_roundtrip_and_ring_plan():
    h = _runtime.encode_frame_header(bytes(range(16)), 7, 1, 31, 2, 5, 0, 1024, 3)
    assert len(h) == 49 and h[44] == 3 and h[45:] == b"\0\0\0\0"
    assert h[16:20] == (7).to_bytes(4, "big")
    d = _runtime.decode_frame_header(h)
    assert d == (bytes(range(16)), 7, 1, 31, 2, 5, 0, 1024, 3)
    with pytest.raises(ValueError):
        _runtime.decode_frame_header(h[:48])
    with pytest.raises(ValueError):
        _runtime.decode_frame_header(h[:44] + b"\x09" + h[45:])
    # reduce-scatter / all-gather chunk bookkeeping for a 3-ring
    assert _runtime.ring_chunk_plan(0, 3, 0, False) == (0, 2)
    assert _runtime.ring_chunk_plan(0, 3, 0, True) == (1, 0)
    assert _runtime.chunk_ranges(10, 3) == [(0, 4), (4, 8), (8, 10)]


# ------------------------------------------------------------------------------------ coordinator
@pytest.fixture(scope="module")
def weights():
    return synthetic_reference_weights(get_preset("tiny"), seed=21)


def _req(prompt, n, temp=0.0, top_p=1.0, interval=0):
    return InferenceRequest(network_id="net", model_id="tiny", prompt_tokens=prompt, executor_id="ex",
                            config=GenerationConfig(max_tokens=n, temperature=temp, top_p=top_p,
                                                    checkpoint_interval=interval))


def test_process_inference_matches_oracle_generate(weights):
    c = InferenceCoordinator(CpuReferenceBackend(weights), EngineConfig(max_decode_batch_size=4))
    r = _req([5, 6, 7, 8], 5)
    res = c.process_inference(r)
    assert res.success and res.completion_tokens == 5
    want = LocalForwardPass(weights).generate([5, 6, 7, 8], 5)
    assert res.generated_tokens == want


def test_sampling_seeded_by_job_and_position(weights):
    r = _req([3, 1, 4, 1, 5], 4, temp=0.8, top_p=0.9)
    a = InferenceCoordinator(CpuReferenceBackend(weights)).process_inference(r)
    want = LocalForwardPass(weights).generate([3, 1, 4, 1, 5], 4, temperature=0.8, top_p=0.9,
                                             seed_base=r.seed_for_position(0))
    assert a.generated_tokens == want


def test_concurrent_sessions_batch_and_each_matches_alone(weights):
    cfg = EngineConfig(max_decode_batch_size=3)
    c = InferenceCoordinator(CpuReferenceBackend(weights), cfg)
    prompts = [[1, 2, 3], [9, 8, 7, 6], [4, 4], [10, 11, 12, 13, 14]]
    reqs = [_req(p, 4) for p in prompts]
    for r in reqs:
        c.submit(r)
    results = {r.job_id: r for r in c.run_until_idle()}
    assert len(results) == 4
    assert c.stats.get("decode_batch_size_peak") == 3
    assert c.stats.get("decode_batch_capacity_deferrals") >= 1
    for r, p in zip(reqs, prompts):
        assert results[r.job_id].generated_tokens == LocalForwardPass(weights).generate(p, 4)


def test_segments_prefill_then_decode(weights):
    c = InferenceCoordinator(CpuReferenceBackend(weights))
    r = _req([2, 7, 1, 8], 6)
    pc = c.process_segment(r)
    assert isinstance(pc, PrefillComplete) and pc.kv_cache_seq_len == 4 and pc.completion_tokens == 1
    r.phase = ExecutionPhase.DECODE
    res = c.process_segment(r)
    assert res.generated_tokens == LocalForwardPass(weights).generate([2, 7, 1, 8], 6)


def test_checkpoint_export_hydrate_continues_identically(weights, tmp_path):
    cm = CheckpointManager(CheckpointConfig(checkpoint_dir=tmp_path))
    c = InferenceCoordinator(CpuReferenceBackend(weights), checkpoints=cm, worker_id="w0")
    r = _req([6, 5, 4, 3, 2], 8, interval=3)
    c.submit(r)
    for _ in range(5):  # prefill + 4 decode steps
        c.step()
    blob = c.export_session_checkpoint_bytes(r.session_id)
    assert c.stats.get("checkpoints_created") >= 1
    assert cm.load(r.job_id) is not None
    # a second worker resumes from the checkpoint bytes
    c2 = InferenceCoordinator(CpuReferenceBackend(weights), worker_id="w1")
    sid = c2.hydrate_session(blob)
    res = c2.run_until_idle()
    assert len(res) == 1 and res[0].recovered_from_checkpoint
    assert res[0].generated_tokens == LocalForwardPass(weights).generate([6, 5, 4, 3, 2], 8)
    # the governor blocks an immediate second restore of the same session
    with pytest.raises(RuntimeError):
        c2.hydrate_session(blob)


def test_pause_resume_and_evict(weights):
    c = InferenceCoordinator(CpuReferenceBackend(weights), EngineConfig(max_decode_batch_size=4))
    a, b = _req([1, 2], 4), _req([3, 4], 4)
    c.submit(a)
    c.submit(b)
    c.step()
    c.step()  # both prefilled
    c.pause_session(a.session_id, SessionPauseReason.REGROUP)
    c.step()
    assert len(c.sessions[a.session_id].generated) == 1 and len(c.sessions[b.session_id].generated) == 2
    c.resume_session(a.session_id)
    blob = c.evict_session(b.session_id, __import__("mesh_b200.engine.types", fromlist=["x"]).SessionEvictionReason.IDLE_SESSION)
    assert blob and c.sessions[b.session_id].status == SessionRuntimeStatus.EVICTED
    res = c.run_until_idle()
    assert [x.job_id for x in res] == [a.job_id]


def test_recovery_governor():
    g = RecoveryGovernor(cooldown_s=5, max_loads_per_minute=2)
    assert g.check("s", 0.0) is None
    g.record("s", 0.0)
    assert g.check("s", 1.0) == "cooldown"
    g.record("t", 2.0)
    assert g.check("u", 3.0) == "budget"
    assert g.check("u", 61.0) is None


def test_checkpoint_manager_retention_and_hash(tmp_path):
    cm = CheckpointManager(CheckpointConfig(checkpoint_dir=tmp_path, max_checkpoints_per_job=2))
    for i in range(4):
        cm.save(Checkpoint.new("job", i, {"a": 1}, [1, 2, i], {"max_tokens": 3}))
    metas = cm.list("job")
    assert [m.token_index for m in metas] == [2, 3]
    cp = cm.load("job")
    assert cp.generated_tokens == [1, 2, 3]
    raw = bytearray((tmp_path / "job" / f"{cp.metadata.checkpoint_id}.ckpt").read_bytes())
    import cbor2
    d = cbor2.loads(bytes(raw))
    d["generated_tokens"] = [9, 9, 9]
    with pytest.raises(ValueError):
        Checkpoint.from_bytes(cbor2.dumps(d))


def test_checkpoint_manager_reads_reference_named_files(tmp_path):
    """A checkpoint written the reference's way (``<job>/<id>.ckpt``) is listed and loaded, and a
    leftover temp file of an interrupted write is ignored."""
    cm = CheckpointManager(CheckpointConfig(checkpoint_dir=tmp_path))
    cp = Checkpoint.new("job-r", 7, {"prompt": "x"}, [5, 6], {"max_tokens": 8})
    (tmp_path / "job-r").mkdir()
    (tmp_path / "job-r" / f"{cp.metadata.checkpoint_id}.ckpt").write_bytes(cp.to_bytes())
    (tmp_path / "job-r" / "partial.ckpt.tmp").write_bytes(b"garbage")
    metas = cm.list("job-r")
    assert [m.checkpoint_id for m in metas] == [cp.metadata.checkpoint_id]
    got = cm.load("job-r")
    assert got.generated_tokens == [5, 6] and got.metadata.token_index == 7
    saved = cm.save(Checkpoint.new("job-r", 9, {}, [5, 6, 7], {}))
    assert saved.suffix == ".ckpt" and not list((tmp_path / "job-r").glob("*.cbor"))


def test_stats_keys_and_persist(tmp_path):
    s = InferenceStats()
    s.add("jobs_completed")
    s.add("decode_batch_size_peak", 4)
    s.add("decode_batch_size_peak", 2)
    assert s.get("decode_batch_size_peak") == 4
    p = s.save_to_file(str(tmp_path))
    back = InferenceStats.load(p)
    assert back.get("jobs_completed") == 1
    assert "avg_tokens_per_second" in s.snapshot()


def test_token_ceiling_buckets():
    assert token_ceiling(100) == 2048 and token_ceiling(2049) == 8192 and token_ceiling(10 ** 6) == -1
