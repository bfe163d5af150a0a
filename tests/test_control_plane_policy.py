"""Behaviour of the control plane's planning, scheduling, failover and provider-contract logic.

Each test restates a behaviour the reference control plane pins with a unit test of the same
subject (``control-plane/src/services/{scheduler,planner,failover}.rs``, ``model_assets.rs``,
``provider.rs``); names follow those behaviours. Pure functions, CPU only.
"""
import pytest

from mesh_b200.control_plane import failover as fo
from mesh_b200.control_plane import planner as pl
from mesh_b200.control_plane import scheduler as sc
from mesh_b200.control_plane.layout import LayoutError, LayoutRule, Member, ModelManifest, validate_group
from mesh_b200.control_plane.provider import BackendContractDescriptor, VerifiedRuntimeCapabilities

NOW = "2026-04-25T12:00:00Z"
CUDA = BackendContractDescriptor.for_provider("cuda")
CPU = BackendContractDescriptor.for_provider("cpu")


# ---------------------------------------------------------------------------------------------- helpers
def manifest(dim=100, heads=None, kv=None, total=1 << 30, layers=None, prefill=(), decode=()):
    return ModelManifest("m", dim, heads, kv, total, layers, tuple(prefill), tuple(decode))


def mem(dev, a, b, pos=0, cap=4, contract=CUDA, memory=0, **kw):
    return Member(dev, pos, a, b, contributed_memory=memory, assigned_capacity_units=cap, backend_contract=contract,
                  **kw)


def cand(aid, phase="decode", status="decode_ready", q="ready", **kw):
    kw.setdefault("created_at", "2026-04-25T11:00:00Z")
    kw.setdefault("decode_ready_at", "2026-04-25T11:30:00Z" if phase == "decode" else None)
    return sc.Candidate(assignment_id=aid, job_id="j-" + aid, session_id="s-" + aid, phase=phase,
                        group_status=status, decode_queue_status=q if phase == "decode" else None, **kw)


def pick(cands, mode="fit_first", dev="worker-1", snap=None, pol=None):
    return sc.schedule(cands, dev, NOW, mode, pol, snap).selected_assignment_id


# ---------------------------------------------------------------------------------------------- scheduler
def test_blocked_decode_transfer_is_reported():
    d = sc.schedule([cand("a", q="blocked_on_transfer")], "w", NOW)
    assert d.selected_assignment_id is None and d.blocked[0].reason == "waiting_for_transfer"


def test_decode_without_queue_row_is_queue_missing():
    d = sc.schedule([cand("a", q=None)], "w", NOW)
    assert d.blocked[0].reason == "queue_missing"


def test_fresh_decode_waits_for_blocked_prefill_siblings_to_form_cohort():
    c = cand("a", decode_cohort_ready_sessions=1, decode_cohort_blocked_sessions=2,
             decode_cohort_blocked_prefill_sessions=2)
    d = sc.schedule([c], "w", NOW)
    assert d.blocked[0].reason == "waiting_for_prefill_cohort"


def test_fresh_decode_does_not_wait_for_transfer_blocked_siblings():
    c = cand("a", decode_cohort_ready_sessions=1, decode_cohort_blocked_sessions=2,
             decode_cohort_blocked_prefill_sessions=0)
    assert pick([c]) == "a"


def test_decode_stops_waiting_once_cohort_has_a_lease():
    c = cand("a", decode_cohort_ready_sessions=1, decode_cohort_blocked_prefill_sessions=1,
             decode_cohort_blocked_sessions=1, decode_cohort_leased_sessions=1)
    assert pick([c]) == "a"


def test_latency_prefers_older_ready_decode_work():
    old = cand("old", decode_ready_at="2026-04-25T11:00:00Z")
    new = cand("new", decode_ready_at="2026-04-25T11:50:00Z")
    assert pick([new, old], "latency_first") == "old"


def test_runtime_mode_priority_latency_before_fit_first():
    a = cand("fit", runtime_mode="fit_first")
    b = cand("lat", runtime_mode="latency_first")
    assert pick([a, b]) == "lat"
    assert [sc.runtime_mode_priority(m) for m in sc.MODES] == [3, 2, 0, 1]


def test_throughput_prefers_better_topology_when_queue_state_ties():
    a = sc.Runnable(cand("efficient", decode_topology_rank=100), NOW)
    b = sc.Runnable(cand("broad", decode_topology_rank=10_000), NOW)
    assert sc.topology_rank("throughput_first", a) < sc.topology_rank("throughput_first", b)
    # other modes ignore the topology rank
    assert sc.topology_rank("latency_first", a) == sc.topology_rank("latency_first", b) == 0


def test_fit_first_respects_submitter_soft_cap_before_arrival_order():
    busy = cand("busy", submitted_by_device_id="alice", created_at="2026-04-25T10:00:00Z")
    idle = cand("idle", submitted_by_device_id="bob", created_at="2026-04-25T11:00:00Z")
    snap = sc.Snapshot(active_jobs_by_submitter={"alice": 1}, online_worker_count=4, online_capacity_units=16)
    assert pick([busy, idle], snap=snap) == "idle"
    assert pick([busy, idle]) == "busy"


def test_model_soft_cap_demotes_a_saturated_model():
    hot = cand("hot", model_id="big")
    cold = cand("cold", model_id="small")
    snap = sc.Snapshot(active_jobs_by_model={"big": 2}, online_worker_count=4, online_capacity_units=64)
    assert pick([hot, cold], snap=snap) == "cold"


def test_fit_first_finishes_inflight_prefill_group_before_fresh_work():
    fresh = cand("fresh", "prefill", "prefill_member", created_at="2026-04-25T09:00:00Z")
    infl = cand("infl", "prefill", "prefill_member", prefill_group_total_members=2, prefill_group_leased_members=1,
                created_at="2026-04-25T11:00:00Z")
    assert pick([fresh, infl]) == "infl"


def test_fresh_prefill_blocked_while_same_model_prefill_group_inflight():
    c = cand("p", "prefill", "prefill_member", model_prefill_inflight_groups=1)
    assert sc.schedule([c], "w", NOW).blocked[0].reason == "lease_held_by_peer"


def test_fresh_prefill_requires_group_leader_to_open_new_cohort():
    follower = cand("p", "prefill", "prefill_member", ring_position=1)
    leader = cand("q", "prefill", "prefill_member", ring_position=0)
    d = sc.schedule([follower, leader], "w", NOW)
    assert d.selected_assignment_id == "q" and d.blocked[0].reason == "lease_held_by_peer"


def test_active_prefill_member_is_already_running():
    assert sc.schedule([cand("p", "prefill", "prefill_active")], "w", NOW).blocked[0].reason == "already_running"


def test_fresh_prefill_blocked_by_foreign_transport_island_job():
    c = cand("p", "prefill", "prefill_member", foreign_transport_island_inflight_jobs=1)
    assert sc.schedule([c], "w", NOW).blocked[0].reason == "lease_held_by_peer"


def test_inflight_prefill_member_attaches_despite_foreign_island_pressure():
    c = cand("p", "prefill", "prefill_member", foreign_transport_island_inflight_jobs=1,
             prefill_group_total_members=2, prefill_group_active_members=1)
    assert pick([c]) == "p"


def test_fresh_decode_blocked_while_peer_prefill_group_inflight():
    c = cand("d", model_prefill_inflight_groups=1)
    assert sc.schedule([c], "w", NOW).blocked[0].reason == "lease_held_by_peer"


def test_fresh_decode_blocked_while_peer_decode_cohort_active():
    c = cand("d", decode_cohort_active_sessions=1)
    assert sc.schedule([c], "w", NOW).blocked[0].reason == "lease_held_by_peer"


def test_decode_member_can_join_peer_owned_leased_cohort():
    c = cand("d", status="decode_member", q="leased", decode_lease_owner_device_id="peer",
             decode_lease_expires_at="2026-04-25T12:01:00Z", decode_cohort_leased_sessions=1)
    assert pick([c], dev="me") == "d"


def test_peer_lease_blocks_non_attachable_decode_state():
    c = cand("d", status="decode_pending", q="leased", decode_lease_owner_device_id="peer",
             decode_lease_expires_at="2026-04-25T12:01:00Z")
    assert sc.schedule([c], "me", NOW).blocked[0].reason == "lease_held_by_peer"


def test_decode_ready_can_join_peer_owned_active_cohort():
    c = cand("d", status="decode_ready", q="active", group_lease_owner_device_id="peer")
    assert pick([c], dev="me") == "d"


def test_own_active_decode_is_already_running():
    c = cand("d", status="decode_active", q="active", group_lease_owner_device_id="me")
    assert sc.schedule([c], "me", NOW).blocked[0].reason == "already_running"


def test_latency_prefers_filling_owned_group_before_fresh_ready_group():
    owned = cand("owned", status="decode_member", group_lease_owner_device_id="me", decode_lease_target_session_count=4,
                 decode_cohort_leased_sessions=2, decode_cohort_ready_sessions=1)
    fresh = cand("fresh", decode_cohort_ready_sessions=8, decode_ready_at="2026-04-25T10:00:00Z")
    assert pick([fresh, owned], "latency_first", dev="me") == "owned"


def test_latency_opens_fresh_group_once_owned_group_reaches_target():
    owned = cand("owned", status="decode_member", group_lease_owner_device_id="me", decode_lease_target_session_count=2,
                 decode_cohort_leased_sessions=2)
    fresh = cand("fresh", decode_cohort_ready_sessions=4)
    assert pick([owned, fresh], "latency_first", dev="me") == "fresh"


def test_throughput_prefers_larger_fresh_cohort_while_latency_prefers_ready_runway():
    big = cand("big", decode_lease_target_session_count=8, decode_cohort_ready_sessions=2)
    ready = cand("ready", decode_lease_target_session_count=2, decode_cohort_ready_sessions=6)
    assert pick([big, ready], "throughput_first") == "big"
    assert pick([big, ready], "latency_first") == "ready"


def test_fit_first_prefers_smaller_fresh_cohort_while_throughput_prefers_larger():
    small = cand("small", decode_lease_target_session_count=2, decode_cohort_ready_sessions=2)
    large = cand("large", decode_lease_target_session_count=8, decode_cohort_ready_sessions=2)
    assert pick([small, large], "fit_first") == "small"
    assert pick([small, large], "throughput_first") == "large"


def test_resilient_edge_prefers_lower_transfer_debt_fresh_cohort():
    debt = cand("debt", decode_cohort_blocked_sessions=5, decode_cohort_ready_sessions=9)
    clean = cand("clean", decode_cohort_blocked_sessions=0, decode_cohort_ready_sessions=1)
    assert pick([debt, clean], "resilient_edge") == "clean"


def test_throughput_drains_leased_owned_decode_before_fresh_group():
    leased = cand("leased", status="decode_leased", q="leased", group_lease_owner_device_id="me",
                  decode_lease_owner_device_id="me", decode_lease_target_session_count=4,
                  decode_cohort_leased_sessions=4)
    fresh = cand("fresh", decode_cohort_ready_sessions=8, decode_lease_target_session_count=8)
    assert pick([fresh, leased], "throughput_first", dev="me") == "leased"


def test_resilient_edge_prefers_fresh_ready_decode_before_leased_owned():
    leased = cand("leased", status="decode_leased", q="leased", group_lease_owner_device_id="me",
                  decode_lease_owner_device_id="me", decode_cohort_leased_sessions=1)
    fresh = cand("fresh")
    assert pick([leased, fresh], "resilient_edge", dev="me") == "fresh"


def test_claim_order_inflight_prefill_then_waiting_decode_cohort_then_rank():
    dec = cand("dec")
    pre_new = cand("pnew", "prefill", "prefill_member", created_at="2026-04-25T11:10:00Z")
    pre_wait = cand("pwait", "prefill", "prefill_member", created_at="2026-04-25T11:20:00Z")
    d = sc.select_claim([dec, pre_new, pre_wait], "w", NOW, waiting_decode_cohort={"pwait": "2026-04-25T09:00:00Z"})
    assert d.selected_assignment_id == "pwait"
    pre_inflight = cand("pin", "prefill", "prefill_leased", prefill_group_leased_members=1,
                        prefill_group_total_members=2)
    d = sc.select_claim([dec, pre_wait, pre_inflight], "w", NOW, waiting_decode_cohort={"pwait": NOW})
    assert d.selected_assignment_id == "pin"


def test_unknown_scheduler_mode_is_rejected():
    with pytest.raises(ValueError):
        sc.schedule([cand("a")], "w", NOW, "fastest")


# ---------------------------------------------------------------------------------------------- layouts
def test_tensor_parallel_group_must_tile_columns_aligned_to_gqa_width():
    m = manifest(dim=4096, heads=32, kv=8)  # GQA width 4 * 128 = 512
    ok = [mem("a", 0, 2048, 0), mem("b", 2048, 4096, 1)]
    assert validate_group(m, "prefill", ok).tensor_parallel_degree == 2
    with pytest.raises(LayoutError, match="aligned"):
        validate_group(m, "prefill", [mem("a", 0, 2000, 0), mem("b", 2000, 4096, 1)])
    with pytest.raises(LayoutError, match="gap"):
        validate_group(m, "prefill", [mem("a", 0, 1024, 0), mem("b", 2048, 4096, 1)])
    with pytest.raises(LayoutError, match="overlaps"):
        validate_group(m, "prefill", [mem("a", 0, 3072, 0), mem("b", 2048, 4096, 1)])


def test_default_decode_rules_prefer_full_replica_then_tensor_parallel():
    m = manifest()
    assert validate_group(m, "decode", [mem("a", 0, 100)]).layout == "full_replica"
    assert validate_group(m, "decode", [mem("a", 0, 50, 0), mem("b", 50, 100, 1)]).layout == "tensor_parallel"


def test_pipeline_rule_needs_full_replicas_and_exact_degree():
    stages = [{"stage_index": 0, "layer_start": 0, "layer_end": 4}, {"stage_index": 1, "layer_start": 4, "layer_end": 8}]
    m = ModelManifest.from_json({"model_id": "m", "tensor_parallelism_dim": 100, "total_model_bytes": 1,
                                 "transformer_layer_count": 8,
                                 "execution_layout": {"decode": [{"layout": "pipeline", "pipeline_parallel_degree": 2,
                                                                  "pipeline_stages": stages}]}})
    r = validate_group(m, "decode", [mem("a", 0, 100, 0), mem("b", 0, 100, 1)])
    assert r.pipeline_parallel_degree == 2 and len(r.pipeline_stages) == 2
    with pytest.raises(LayoutError):
        validate_group(m, "decode", [mem("a", 0, 100, 0)])


def test_invalid_pipeline_partition_metadata_is_rejected():
    bad = [{"stage_index": 0, "layer_start": 0, "layer_end": 3}, {"stage_index": 1, "layer_start": 4, "layer_end": 8}]
    with pytest.raises(LayoutError, match="expected 3"):
        ModelManifest.from_json({"model_id": "m", "tensor_parallelism_dim": 100, "transformer_layer_count": 8,
                                 "execution_layout": {"decode": [{"layout": "pipeline", "pipeline_parallel_degree": 2,
                                                                  "pipeline_stages": bad}]}})
    with pytest.raises(LayoutError, match="pipeline_parallel_degree"):
        ModelManifest.from_json({"model_id": "m", "tensor_parallelism_dim": 100,
                                 "execution_layout": {"prefill": [{"layout": "tensor_pipeline_hybrid",
                                                                   "tensor_parallel_degree": 2}]}})
    with pytest.raises(LayoutError, match="min_members"):
        ModelManifest.from_json({"model_id": "m", "tensor_parallelism_dim": 100,
                                 "execution_layout": {"decode": [{"layout": "full_replica", "min_members": 0}]}})


def test_hybrid_layout_checks_each_stage_tiles_the_columns():
    rule = LayoutRule("tensor_pipeline_hybrid", tensor_parallel_degree=2, pipeline_parallel_degree=2,
                      pipeline_stages=())
    m = manifest(decode=[rule], layers=4)
    good = [mem("a", 0, 50, 0), mem("b", 50, 100, 1), mem("c", 0, 50, 2), mem("d", 50, 100, 3)]
    assert validate_group(m, "decode", good).tensor_parallel_degree == 2
    bad = [mem("a", 0, 50, 0), mem("c", 0, 50, 1), mem("b", 50, 100, 2), mem("d", 50, 100, 3)]
    with pytest.raises(LayoutError):
        validate_group(m, "decode", bad)


def test_provider_constraints_and_homogeneity():
    rule = LayoutRule("tensor_parallel", allowed_providers=("cuda",), requires_homogeneous=True)
    m = manifest(prefill=[rule])
    with pytest.raises(LayoutError, match="allowed providers"):
        validate_group(m, "prefill", [mem("a", 0, 50, 0), mem("b", 50, 100, 1, contract=CPU)])
    other = BackendContractDescriptor.for_provider("cuda", "cuda_fused")
    with pytest.raises(LayoutError, match="homogeneous"):
        validate_group(m, "prefill", [mem("a", 0, 50, 0), mem("b", 50, 100, 1, contract=other)])


# ---------------------------------------------------------------------------------------------- planner
def _ring(*spans, caps=None):
    caps = caps or [4] * len(spans)
    return [mem(f"w{i}", a, b, i, caps[i]) for i, (a, b) in enumerate(spans)]


def test_planner_builds_tensor_parallel_prefill_and_co_located_decode():
    ms = _ring((0, 50), (50, 100))
    p = pl.plan(manifest(), ms)
    assert [m.device_id for m in p.prefill] == ["w0", "w1"]
    assert [m.device_id for m in p.decode] == ["w0", "w1"]
    assert p.kv_transfer_policy == "co_located"
    j = p.to_json("m", "sess")
    assert j["execution_groups"][0]["group_id"] == f"group-{p.plan_id}-prefill"
    assert j["segments"][1]["segment_id"] == "segment-sess-decode"


def test_planner_shrinks_decode_to_a_full_replica_and_hands_kv_off():
    ms = _ring((0, 50), (50, 100)) + [mem("full", 0, 100, 2, 8)]
    p = pl.plan(manifest(), ms)
    assert [m.device_id for m in p.decode] == ["full"]
    assert p.kv_transfer_policy == "checkpoint_handoff"


def test_planner_skips_workers_without_production_contract():
    weak = BackendContractDescriptor("cuda", "cuda_fast_path", "x", False, True, True, True, True, "discrete_vram",
                                     verified_runtime=VerifiedRuntimeCapabilities(True, True, True, True, True)).with_hash()
    ms = [mem("w0", 0, 100, 0, contract=weak)]
    with pytest.raises(pl.PlanningError):
        pl.plan(manifest(), ms)


def test_planner_accepts_cpu_only_topology():
    ms = [mem("c0", 0, 50, 0, contract=CPU), mem("c1", 50, 100, 1, contract=CPU)]
    p = pl.plan(manifest(), ms)
    assert p.prefill_island.startswith("island:m:prefill:cpu_portable:")


def test_planner_selects_valid_provider_constrained_variant_when_first_is_illegal():
    rules = [LayoutRule("full_replica", "cpu_only", allowed_providers=("cpu",)), LayoutRule("tensor_parallel")]
    m = manifest(decode=rules)
    p = pl.plan(m, _ring((0, 50), (50, 100)))
    assert len(p.decode) == 2


def test_planner_refuses_decode_group_when_provider_constraints_fail():
    m = manifest(decode=[LayoutRule("tensor_parallel", allowed_providers=("metal",))])
    with pytest.raises(pl.PlanningError, match="decode"):
        pl.plan(m, _ring((0, 50), (50, 100)))


def test_runtime_mode_follows_connectivity_and_capacity_spread():
    assert pl.derive_runtime_mode(_ring((0, 100))) == "latency_first"
    assert pl.derive_runtime_mode(_ring((0, 50), (50, 100), caps=[1, 8])) == "throughput_first"
    relayed = [mem("r", 0, 100, 0, active_path="relay")]
    assert pl.derive_runtime_mode(relayed) == "resilient_edge"


def test_topology_efficiency_penalises_broad_imbalanced_groups():
    balanced = _ring((0, 50), (50, 100), caps=[4, 4])
    broad = _ring((0, 25), (25, 50), (50, 75), (75, 100), caps=[1, 16, 1, 16])
    assert pl.topology_efficiency_score(balanced, "latency_first") > pl.topology_efficiency_score(broad, "latency_first")


def test_kv_owner_has_most_capacity_then_memory_then_lowest_position():
    ms = [mem("a", 0, 50, 0, 4, memory=1), mem("b", 50, 100, 1, 4, memory=2), mem("c", 0, 100, 2, 2)]
    assert pl.select_kv_owner(ms) == "b"
    assert pl.select_kv_owner([mem("x", 0, 1, 3), mem("y", 0, 1, 1)]) == "y"


def test_refresh_decode_plan_keeps_unchanged_participants():
    ms = _ring((0, 50), (50, 100))
    p = pl.plan(manifest(), ms)
    q = pl.refresh_decode_plan(manifest(), p, ms)
    assert [m.device_id for m in q.decode] == [m.device_id for m in p.decode]


def test_refresh_decode_plan_needs_a_material_gain_to_move():
    ms = _ring((0, 50), (50, 100))
    p = pl.plan(manifest(), ms)
    # a new full replica of equal capacity appears: not better by the margin, keep the current group
    q = pl.refresh_decode_plan(manifest(), p, ms + [mem("full", 0, 100, 2, 4)])
    assert [m.device_id for m in q.decode] == ["w0", "w1"]
    # a strong full replica is materially better: move the decode group there
    q = pl.refresh_decode_plan(manifest(), p, ms + [mem("full", 0, 100, 2, 64)])
    assert [m.device_id for m in q.decode] == ["full"]


def test_refresh_decode_plan_refuses_when_no_valid_regroup():
    ms = _ring((0, 50), (50, 100))
    p = pl.plan(manifest(), ms)
    with pytest.raises(pl.PlanningError):
        pl.refresh_decode_plan(manifest(), p, ms[:1])


# ---------------------------------------------------------------------------------------------- failover
def _dec_session(parts, owner="w0", ckpt=None):
    return fo.SessionView("s", "decode_active", "decode", parts, owner, 10, ckpt, "t0" if ckpt else None, "seg-d")


def test_failover_healthy_when_losses_miss_active_participants():
    grp = _ring((0, 50), (50, 100), (50, 100))
    d = fo.FailoverEngine().evaluate(_dec_session(["w0", "w1"]), grp, ["w2"])
    assert d.recovery_state == "healthy" and d.strategy == "none"


def test_failover_fails_prefill_on_participant_loss():
    s = fo.SessionView("s", "prefill_active", "prefill", ["w0", "w1"], "w0")
    d = fo.FailoverEngine().evaluate(s, _ring((0, 50), (50, 100)), ["w1"])
    assert d.recovery_state == "failed" and d.resume_mode == "manual_intervention"


def test_failover_shrinks_decode_when_survivors_cover_the_span():
    grp = [mem("w0", 0, 100, 0), mem("w1", 50, 100, 1)]
    d = fo.FailoverEngine().evaluate(_dec_session(["w0", "w1"]), grp, ["w1"], "active")
    assert d.strategy == "shrink" and d.resume_mode == "immediate" and d.recovery_state == "resume_ready"
    assert d.target_participant_device_ids == ["w0"] and d.decode_queue_status == "ready" and d.pause_required


def test_failover_replacement_pauses_for_checkpoint_transfer():
    grp = _ring((0, 50), (50, 100), (50, 100))
    s = _dec_session(["w0", "w1"], ckpt="w0")
    d = fo.FailoverEngine().evaluate(s, grp, ["w1"])
    assert d.strategy == "replace" and d.replacement_device_ids == ["w2"]
    assert d.resume_mode == "requires_checkpoint_transfer" and d.recovery_state == "paused"
    assert d.decode_queue_status == "blocked_on_transfer" and d.transfer_source_device_id == "w0"


def test_failover_replacement_uses_live_kv_handoff_when_recovery_contract_exists():
    grp = _ring((0, 50), (50, 100), (50, 100))
    sup = fo.SupportGroups(kv={"w0"}, recovery={"w0", "w2"})
    d = fo.FailoverEngine().evaluate(_dec_session(["w0", "w1"]), grp, ["w1"], support=sup)
    assert d.resume_mode == "requires_live_kv_transfer" and d.recovery_state == "paused"


def test_failover_replaces_without_pause_after_completed_live_handoff():
    grp = _ring((0, 50), (50, 100), (50, 100))
    t = fo.KvTransfer("seg-d", "w0", "w2", "live_kv_handoff", "completed", 12)
    d = fo.FailoverEngine().evaluate(_dec_session(["w0", "w1"]), grp, ["w1"], transfers=[t])
    assert d.resume_mode == "immediate" and d.strategy == "replace" and d.recovery_state == "resume_ready"


def test_failover_fails_decode_when_replacement_needs_missing_checkpoint():
    grp = _ring((0, 50), (50, 100), (50, 100))
    d = fo.FailoverEngine().evaluate(_dec_session(["w0", "w1"]), grp, ["w1"])
    assert d.recovery_state == "failed" and "no checkpoint" in d.reason


def test_failover_fails_when_nobody_covers_the_span():
    grp = _ring((0, 50), (50, 100))
    d = fo.FailoverEngine().evaluate(_dec_session(["w0", "w1"], ckpt="w0"), grp, ["w1"])
    assert d.recovery_state == "failed" and "cover" in d.reason


def test_failover_four_worker_ring_shrinks_to_three():
    grp = [mem("w0", 0, 25, 0), mem("w1", 25, 50, 1), mem("w2", 50, 100, 2), mem("w3", 75, 100, 3)]
    d = fo.FailoverEngine().evaluate(_dec_session(["w0", "w1", "w2", "w3"]), grp, ["w3"])
    assert d.strategy == "shrink" and d.target_participant_device_ids == ["w0", "w1", "w2"]


def test_covers_required_span_rejects_one_column_gap():
    ms = {m.device_id: m for m in [mem("a", 0, 49), mem("b", 50, 100)]}
    assert not fo.covers_required_span(ms, ["a", "b"], (0, 100))
    ms["a"] = mem("a", 0, 50)
    assert fo.covers_required_span(ms, ["a", "b"], (0, 100))


def test_next_kv_owner_prefers_newest_kv_when_owner_is_lost():
    grp = _ring((0, 50), (50, 100), (0, 50), (50, 100))
    s = _dec_session(["w0", "w1"], owner="w1", ckpt="w0")
    d = fo.FailoverEngine().evaluate(s, grp, ["w1"], kv_positions={"w3": 9})
    assert d.next_kv_owner_device_id in d.target_participant_device_ids
    assert d.transfer_source_device_id == "w0"  # the owner is lost: the checkpoint holder sends


# ---------------------------------------------------------------------------------------------- provider
def test_provider_contract_hash_is_stable_and_distinguishes_profiles():
    a = BackendContractDescriptor.for_provider("cuda")
    b = BackendContractDescriptor.for_provider("cuda")
    assert a.contract_hash == b.contract_hash and len(a.contract_hash) == 16 and a.hash_is_current()
    assert a.optimization_profile == "b200_fused"
    assert BackendContractDescriptor.for_provider("cuda", "cuda_fused").contract_hash != a.contract_hash
    assert BackendContractDescriptor.from_json(a.to_json()) == a


def test_provider_contract_runtime_consistency():
    BackendContractDescriptor.for_provider("cpu").validate_runtime_consistency()
    bad = BackendContractDescriptor("cpu", "cpu_portable", "p", True, True, True, True, True, "system_ram",
                                    verified_runtime=VerifiedRuntimeCapabilities(True, True, True, True, False))
    with pytest.raises(ValueError, match="device sampling"):
        bad.validate_runtime_consistency()
    assert not BackendContractDescriptor.for_provider("cpu").supports_device_sampling
    with pytest.raises(ValueError):
        BackendContractDescriptor.for_provider("rocm")


# --------------------------------------------------------------------------- device certificates
def test_certificate_issue_verify_tamper_and_expiry(tmp_path):
    import datetime
    import cbor2
    from mesh_b200.control_plane.certificate import CertificateError, ControlPlaneKeypair, verify_certificate
    kp = ControlPlaneKeypair.load_or_generate(tmp_path / "cp.key")
    assert ControlPlaneKeypair.load_or_generate(tmp_path / "cp.key").public_key() == kp.public_key()  # persisted
    pk = bytes(range(32))
    t0 = datetime.datetime(2026, 1, 1, tzinfo=datetime.timezone.utc)
    blob = kp.generate_certificate("dev-1", "net-1", pk, now=t0)
    cert = kp.verify_certificate(blob)
    assert (cert.device_id, cert.network_id, cert.public_key) == ("dev-1", "net-1", pk)
    assert cert.issued_at == "2026-01-01T00:00:00Z" and cert.expires_at == "2026-01-31T00:00:00Z"
    assert not cert.expired(t0 + datetime.timedelta(days=29)) and cert.expired(t0 + datetime.timedelta(days=30))
    outer = cbor2.loads(blob)
    inner = cbor2.loads(outer["certificate"])
    inner["device_id"] = "dev-2"
    forged = cbor2.dumps({"certificate": cbor2.dumps(inner), "signature": outer["signature"]})
    with pytest.raises(CertificateError):
        kp.verify_certificate(forged)
    with pytest.raises(CertificateError):
        verify_certificate(blob, ControlPlaneKeypair.generate().public_key())
    with pytest.raises(CertificateError):
        kp.generate_certificate("d", "n", b"short")
    with pytest.raises(CertificateError):
        kp.verify_certificate(b"\x00garbage")


def test_registration_issues_certificate_and_validates_inputs():
    from mesh_b200.control_plane.certificate import verify_certificate
    from mesh_b200.control_plane.db import Database
    from mesh_b200.control_plane.service import ApiError, ControlPlane, NotFound
    cp = ControlPlane(Database())
    net = cp.create_network("lan")["network_id"]
    pk = "ab" * 32
    r = cp.register_device("dev-a", net, public_key=pk)
    cert = verify_certificate(bytes.fromhex(r["certificate"]), bytes.fromhex(r["control_plane_public_key"]))
    assert cert.device_id == "dev-a" and cert.network_id == net and cert.public_key.hex() == pk
    stored = cp.db.query("SELECT certificate, public_key FROM devices WHERE device_id=?", ("dev-a",))[0]
    assert stored["certificate"] == r["certificate"] and stored["public_key"] == pk
    assert cp.register_device("dev-b", net)["certificate"] == ""  # no key, no certificate
    with pytest.raises(ApiError):
        cp.register_device("dev-c", net, public_key="ab" * 31)
    with pytest.raises(ApiError):
        cp.register_device("dev-c", net, public_key="zz" * 32)
    with pytest.raises(ApiError):
        cp.register_device("", net)
    with pytest.raises(NotFound):
        cp.register_device("dev-d", "no-such-network")
