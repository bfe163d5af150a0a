"""Model execution layouts: which member groups may serve a phase of a model.

Restates ``control-plane/src/model_assets.rs`` (manifest ``execution_layout``, ``:10-134``; rule
validation ``:250-426``; group validation ``:511-840``):

* a rule names a layout kind: ``tensor_parallel`` (members' column spans tile 0..dim exactly, each
  span aligned to the grouped-query width), ``full_replica`` (every member holds 0..dim),
  ``pipeline`` (full replicas, one per stage, ``pipeline_parallel_degree`` of them) or
  ``tensor_pipeline_hybrid`` (``pp x tp`` members; in ring order, each run of ``tp`` members tiles
  0..dim), optionally with member-count bounds, an exact degree and provider constraints;
* without configured rules, prefill may use any tensor-parallel group and decode prefers a full
  replica, then a tensor-parallel group;
* a group is legal for a phase if it satisfies the first matching rule of that phase.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional, Sequence

from .provider import BackendContractDescriptor

LAYOUT_KINDS = ("tensor_parallel", "full_replica", "pipeline", "tensor_pipeline_hybrid")


class LayoutError(ValueError):
    """An invalid manifest rule (HTTP 400) or an illegal execution group (HTTP 409)."""


@dataclass
class Member:
    """One ring worker as the planner sees it (``api/types.rs`` ExecutionGroupMember)."""
    device_id: str
    ring_position: int
    column_start: int
    column_end: int
    contributed_memory: int = 0
    assigned_capacity_units: int = 1
    backend_contract: BackendContractDescriptor = field(
        default_factory=lambda: BackendContractDescriptor.for_provider("cuda"))
    throughput_multiplier: Optional[float] = None
    observed_tokens_per_second: Optional[float] = None
    observed_deferred_ratio: Optional[float] = None
    observed_fill_ratio: Optional[float] = None
    instability_score: int = 0
    connectivity_status: Optional[str] = "connected"   # connected | degraded | disconnected | None
    active_path: Optional[str] = "direct"              # direct | relay | None
    listen_addrs: List[str] = field(default_factory=lambda: ["dataplane://local"])

    def to_json(self) -> dict:
        return {"device_id": self.device_id, "worker_position": self.ring_position,
                "shard_column_start": self.column_start, "shard_column_end": self.column_end,
                "contributed_memory": self.contributed_memory,
                "assigned_capacity_units": self.assigned_capacity_units,
                "backend_contract_hash": self.backend_contract.contract_hash,
                "provider": self.backend_contract.provider}


@dataclass(frozen=True)
class PipelineStage:
    stage_index: int
    layer_start: int
    layer_end: int


@dataclass(frozen=True)
class LayoutRule:
    layout: str
    variant_name: Optional[str] = None
    min_members: Optional[int] = None
    max_members: Optional[int] = None
    tensor_parallel_degree: Optional[int] = None
    pipeline_parallel_degree: Optional[int] = None
    pipeline_stages: tuple = ()
    allowed_providers: tuple = ()
    requires_homogeneous: bool = False

    @classmethod
    def from_json(cls, d: dict) -> "LayoutRule":
        pc = d.get("provider_constraints") or {}
        stages = tuple(PipelineStage(int(s["stage_index"]), int(s["layer_start"]), int(s["layer_end"]))
                       for s in d.get("pipeline_stages") or [])
        kind = d["layout"]
        if kind not in LAYOUT_KINDS:
            raise LayoutError(f"unknown serving layout {kind!r}")
        return cls(layout=kind, variant_name=d.get("variant_name"), min_members=d.get("min_members"),
                   max_members=d.get("max_members"), tensor_parallel_degree=d.get("tensor_parallel_degree"),
                   pipeline_parallel_degree=d.get("pipeline_parallel_degree"), pipeline_stages=stages,
                   allowed_providers=tuple(pc.get("allowed_providers") or ()),
                   requires_homogeneous=bool(pc.get("requires_homogeneous", False)))


DEFAULT_PREFILL_RULES = (LayoutRule("tensor_parallel", "default_tensor_parallel"),)
DEFAULT_DECODE_RULES = (LayoutRule("full_replica", "default_full_replica"),
                        LayoutRule("tensor_parallel", "default_tensor_parallel"))


@dataclass
class ModelManifest:
    """The parts of ``model.json`` the control plane plans with."""
    model_id: str
    tensor_parallelism_dim: int
    attention_head_count: Optional[int] = None
    kv_head_count: Optional[int] = None
    total_model_bytes: int = 0
    transformer_layer_count: Optional[int] = None
    prefill_rules: tuple = ()
    decode_rules: tuple = ()

    @classmethod
    def from_json(cls, d: dict) -> "ModelManifest":
        lay = d.get("execution_layout") or {}
        m = cls(model_id=d["model_id"], tensor_parallelism_dim=int(d["tensor_parallelism_dim"]),
                attention_head_count=d.get("attention_head_count"), kv_head_count=d.get("kv_head_count"),
                total_model_bytes=int(d.get("total_model_bytes", 0)),
                transformer_layer_count=d.get("transformer_layer_count", d.get("num_layers")),
                prefill_rules=tuple(LayoutRule.from_json(r) for r in lay.get("prefill") or []),
                decode_rules=tuple(LayoutRule.from_json(r) for r in lay.get("decode") or []))
        m.validate_rules()
        return m

    def rules_for(self, phase: str) -> Sequence[LayoutRule]:
        if phase == "prefill":
            return self.prefill_rules or DEFAULT_PREFILL_RULES
        if phase == "decode":
            return self.decode_rules or DEFAULT_DECODE_RULES
        raise LayoutError(f"unknown phase {phase!r}")

    def attention_group_width(self) -> Optional[int]:
        """Columns of one GQA group ((heads / kv_heads) * head_dim), or None without geometry."""
        h, kv = self.attention_head_count, self.kv_head_count
        if h is None or kv is None:
            return None
        if h <= 0 or kv <= 0 or h % kv:
            raise LayoutError(f"model {self.model_id} declares invalid attention geometry num_heads={h} "
                              f"num_kv_heads={kv}")
        if self.tensor_parallelism_dim % h:
            raise LayoutError(f"model {self.model_id} declares tensor_parallelism_dim {self.tensor_parallelism_dim} "
                              f"not divisible by attention_head_count {h}")
        return (h // kv) * (self.tensor_parallelism_dim // h)

    # ------------------------------------------------------------------------------------------
    def validate_rules(self) -> None:
        """Manifest-level checks of every configured rule (``model_assets.rs:250-426``)."""
        for phase, rules in (("prefill", self.prefill_rules), ("decode", self.decode_rules)):
            for i, r in enumerate(rules):
                where = f"{phase} layout rule {i}"
                if r.min_members is not None and r.min_members == 0:
                    raise LayoutError(f"{where} with min_members=0")
                if r.min_members is not None and r.max_members is not None and r.max_members < r.min_members:
                    raise LayoutError(f"{where} with max_members < min_members")
                if r.tensor_parallel_degree is not None and not (
                        0 < r.tensor_parallel_degree <= self.tensor_parallelism_dim):
                    raise LayoutError(f"{where} with invalid tensor_parallel_degree {r.tensor_parallel_degree}")
                if r.layout in ("pipeline", "tensor_pipeline_hybrid"):
                    if r.pipeline_parallel_degree is None:
                        raise LayoutError(f"{where} without pipeline_parallel_degree")
                    if r.pipeline_parallel_degree == 0:
                        raise LayoutError(f"{where} with pipeline_parallel_degree=0")
                    self._validate_stages(where, r.pipeline_parallel_degree, r.pipeline_stages)
                if r.layout == "tensor_pipeline_hybrid" and r.tensor_parallel_degree is None:
                    raise LayoutError(f"{where} without tensor_parallel_degree")
                if r.layout == "pipeline" and r.tensor_parallel_degree is not None:
                    raise LayoutError(f"{where} with unexpected tensor_parallel_degree")

    def _validate_stages(self, where: str, degree: int, stages: Sequence[PipelineStage]) -> None:
        total = self.transformer_layer_count
        if total is None:
            raise LayoutError(f"{where}: pipeline layout without transformer_layer_count")
        if total == 0:
            raise LayoutError(f"{where}: transformer_layer_count=0")
        if len(stages) != degree:
            raise LayoutError(f"{where} with {len(stages)} stage ranges, expected {degree}")
        cursor = 0
        for expected, st in enumerate(sorted(stages, key=lambda s: s.stage_index)):
            if st.stage_index != expected:
                raise LayoutError(f"{where} with non-contiguous stage index {st.stage_index}")
            if st.layer_start >= st.layer_end:
                raise LayoutError(f"{where} stage {st.stage_index} with empty layer range "
                                  f"{st.layer_start}..{st.layer_end}")
            if st.layer_start != cursor:
                raise LayoutError(f"{where} stage {st.stage_index} starting at {st.layer_start}, expected {cursor}")
            cursor = st.layer_end
        if cursor != total:
            raise LayoutError(f"{where} covering layers 0..{cursor}, expected 0..{total}")


@dataclass(frozen=True)
class ResolvedLayout:
    variant_name: Optional[str]
    layout: str
    member_count: int
    tensor_parallel_degree: int
    pipeline_parallel_degree: int
    pipeline_stages: tuple = ()


# ---------------------------------------------------------------------------------------------- groups
def _check_count(members: Sequence[Member], r: LayoutRule) -> None:
    n = len(members)
    if r.min_members is not None and n < r.min_members:
        raise LayoutError(f"requires at least {r.min_members} members, found {n}")
    if r.max_members is not None and n > r.max_members:
        raise LayoutError(f"allows at most {r.max_members} members, found {n}")


def _check_shards(m: ModelManifest, members: Sequence[Member]) -> None:
    dim = m.tensor_parallelism_dim
    for x in members:
        if x.column_start >= x.column_end:
            raise LayoutError(f"member {x.device_id} has an empty shard span {x.column_start}..{x.column_end}")
        if x.column_end > dim:
            raise LayoutError(f"member {x.device_id} shard span {x.column_start}..{x.column_end} exceeds "
                              f"tensor parallel dimension {dim}")


def _check_providers(members: Sequence[Member], r: LayoutRule) -> None:
    if r.allowed_providers:
        for x in members:
            if x.backend_contract.provider not in r.allowed_providers:
                raise LayoutError(f"member {x.device_id} uses provider {x.backend_contract.provider}, allowed "
                                  f"providers are {', '.join(r.allowed_providers)}")
    if r.requires_homogeneous and len({x.backend_contract.contract_hash for x in members}) > 1:
        raise LayoutError("providers must be homogeneous across the group")


def check_tensor_parallel(m: ModelManifest, members: Sequence[Member], degree: Optional[int] = None) -> None:
    if degree is not None and len(members) != degree:
        raise LayoutError(f"requires tensor_parallel_degree={degree}, found {len(members)} members")
    align = m.attention_group_width()
    cursor = 0
    for x in sorted(members, key=lambda x: (x.column_start, x.column_end)):
        if align and (x.column_start % align or x.column_end % align):
            raise LayoutError(f"member {x.device_id} shard span {x.column_start}..{x.column_end} is not aligned to "
                              f"grouped-query width {align}")
        if x.column_start != cursor:
            if x.column_start < cursor:
                raise LayoutError(f"member {x.device_id} overlaps the existing tensor-parallel span at "
                                  f"{x.column_start}..{x.column_end}")
            raise LayoutError(f"tensor-parallel layout leaves a gap before {x.column_start}..{x.column_end}")
        cursor = x.column_end
    if cursor != m.tensor_parallelism_dim:
        raise LayoutError(f"tensor-parallel layout ends at {cursor}, expected {m.tensor_parallelism_dim}")


def check_full_replica(m: ModelManifest, members: Sequence[Member]) -> None:
    for x in members:
        if x.column_start != 0 or x.column_end != m.tensor_parallelism_dim:
            raise LayoutError(f"member {x.device_id} is not a full replica because it serves "
                              f"{x.column_start}..{x.column_end} instead of 0..{m.tensor_parallelism_dim}")


def check_against_rule(m: ModelManifest, members: Sequence[Member], r: LayoutRule) -> ResolvedLayout:
    _check_count(members, r)
    _check_shards(m, members)
    _check_providers(members, r)
    n = len(members)
    if r.layout == "tensor_parallel":
        check_tensor_parallel(m, members, r.tensor_parallel_degree)
        return ResolvedLayout(r.variant_name, r.layout, n, r.tensor_parallel_degree or n, 1)
    if r.layout == "full_replica":
        check_full_replica(m, members)
        return ResolvedLayout(r.variant_name, r.layout, n, 1, 1)
    if r.layout == "pipeline":
        check_full_replica(m, members)
        if r.pipeline_parallel_degree is None:
            raise LayoutError("pipeline layouts require pipeline_parallel_degree")
        if n != r.pipeline_parallel_degree:
            raise LayoutError(f"requires pipeline_parallel_degree={r.pipeline_parallel_degree}, found {n} members")
        return ResolvedLayout(r.variant_name, r.layout, n, 1, r.pipeline_parallel_degree, r.pipeline_stages)
    # tensor_pipeline_hybrid
    pp, tp = r.pipeline_parallel_degree, r.tensor_parallel_degree
    if pp is None:
        raise LayoutError("tensor/pipeline hybrid layouts require pipeline_parallel_degree")
    if tp is None:
        raise LayoutError("tensor/pipeline hybrid layouts require tensor_parallel_degree")
    if n != pp * tp:
        raise LayoutError(f"requires tensor_parallel_degree={tp} and pipeline_parallel_degree={pp}, found {n} members")
    ordered = sorted(members, key=lambda x: x.ring_position)
    for s in range(pp):
        check_tensor_parallel(m, ordered[s * tp:(s + 1) * tp], tp)
    return ResolvedLayout(r.variant_name, r.layout, n, tp, pp, r.pipeline_stages)


def validate_group(m: ModelManifest, phase: str, members: Sequence[Member]) -> ResolvedLayout:
    """The first rule of the phase the group satisfies; LayoutError listing every rule's objection
    otherwise."""
    if not members:
        raise LayoutError("execution group has no members")
    errors = []
    for r in m.rules_for(phase):
        try:
            return check_against_rule(m, members, r)
        except LayoutError as e:
            errors.append(f"{r.layout}: {e}")
    raise LayoutError(f"no legal {phase} layout matched: " + "; ".join(errors))
