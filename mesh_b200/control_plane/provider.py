"""Backend contract descriptors: what an execution provider promises the control plane.

Restates ``control-plane/src/provider.rs:8-216`` (and the agent's copy,
``agent/src/provider/mod.rs:10-356``): a provider kind (cpu / metal / cuda), its compatibility
class, optimisation profile, the serving features it supports and has verified at runtime, its
memory model, and a contract hash that groups interchangeable workers. The planner only forms
execution groups from workers whose contracts support production serving, and an execution
island is a set of workers with one contract hash.

The B200 build's CUDA provider advertises the optimisation profile ``b200_fused`` (the fused
sm_100a kernels) instead of the reference's ``cuda_fused``, so its hash differs from a stock CUDA
worker's and the two never share a fast-path island. The hash is the first 16 hex digits of a
SHA-256 over the canonical JSON of the descriptor's fields (the reference hashes the same fields
with Rust's process-default hasher, which has no portable byte-level definition).
"""
from __future__ import annotations

import hashlib
import json
from dataclasses import asdict, dataclass, field, replace
from typing import Optional

PROVIDERS = ("cpu", "metal", "cuda")
COMPATIBILITY_CLASSES = ("cpu_portable", "metal_fast_path", "cuda_fast_path", "heterogeneous_portable")
MEMORY_MODELS = ("system_ram", "discrete_vram", "unified_memory", "hybrid")


@dataclass(frozen=True)
class VerifiedRuntimeCapabilities:
    fast_path_serving: bool = False
    decode_microbatch: bool = False
    paged_kv: bool = False
    checkpoint_handoff: bool = False
    device_sampling: bool = False


@dataclass(frozen=True)
class BackendContractDescriptor:
    provider: str
    compatibility_class: str
    optimization_profile: str
    supports_decode_microbatch: bool
    supports_paged_kv: bool
    supports_checkpoint_handoff: bool
    supports_device_sampling: bool
    fast_path_eligible: bool
    memory_model: str
    implementation_maturity: str = "verified_fast_path"
    verified_runtime: VerifiedRuntimeCapabilities = field(default_factory=VerifiedRuntimeCapabilities)
    contract_hash: str = ""

    # ------------------------------------------------------------------------------------------
    @classmethod
    def for_provider(cls, provider: str, optimization_profile: Optional[str] = None) -> "BackendContractDescriptor":
        """The descriptor a worker of this provider kind advertises. ``cuda`` on this build is the
        fused sm_100a path (profile ``b200_fused``)."""
        if provider not in PROVIDERS:
            raise ValueError(f"unknown execution provider {provider!r}; expected one of {PROVIDERS}")
        klass = {"cpu": "cpu_portable", "metal": "metal_fast_path", "cuda": "cuda_fast_path"}[provider]
        profile = optimization_profile or {"cpu": "cpu_serial", "metal": "metal_vectorized",
                                           "cuda": "b200_fused"}[provider]
        sampling = provider != "cpu"
        memory = {"cpu": "system_ram", "metal": "unified_memory", "cuda": "discrete_vram"}[provider]
        verified = VerifiedRuntimeCapabilities(fast_path_serving=True, decode_microbatch=True, paged_kv=True,
                                               checkpoint_handoff=True, device_sampling=sampling)
        d = cls(provider=provider, compatibility_class=klass, optimization_profile=profile,
                supports_decode_microbatch=True, supports_paged_kv=True, supports_checkpoint_handoff=True,
                supports_device_sampling=sampling, fast_path_eligible=True, memory_model=memory,
                verified_runtime=verified)
        return d.with_hash()

    def hash_fields(self) -> dict:
        d = asdict(self)
        d.pop("contract_hash")
        return d

    def compute_contract_hash(self) -> str:
        blob = json.dumps(self.hash_fields(), sort_keys=True, separators=(",", ":")).encode()
        return hashlib.sha256(blob).hexdigest()[:16]

    def with_hash(self) -> "BackendContractDescriptor":
        return replace(self, contract_hash=self.compute_contract_hash())

    # ------------------------------------------------------------------------------------------
    def supports_production_serving(self) -> bool:
        v = self.verified_runtime
        return (self.fast_path_eligible and self.supports_decode_microbatch and self.supports_paged_kv and
                v.fast_path_serving and v.decode_microbatch and v.paged_kv)

    def validate_runtime_consistency(self) -> None:
        """Every advertised feature must be runtime-verified (raises ValueError otherwise)."""
        v = self.verified_runtime
        checks = [(self.fast_path_eligible, v.fast_path_serving, "fast-path eligibility"),
                  (self.supports_decode_microbatch, v.decode_microbatch, "decode microbatch"),
                  (self.supports_paged_kv, v.paged_kv, "paged KV"),
                  (self.supports_checkpoint_handoff, v.checkpoint_handoff, "checkpoint handoff"),
                  (self.supports_device_sampling, v.device_sampling, "device sampling")]
        for advertised, verified, what in checks:
            if advertised and not verified:
                raise ValueError(f"provider {self.provider} advertises {what} without runtime verification")

    def hash_is_current(self) -> bool:
        return self.contract_hash == self.compute_contract_hash()

    def to_json(self) -> dict:
        return asdict(self)

    @classmethod
    def from_json(cls, d: dict) -> "BackendContractDescriptor":
        d = dict(d)
        v = d.pop("verified_runtime", {}) or {}
        return cls(verified_runtime=VerifiedRuntimeCapabilities(**v), **d)


def contract_for_device(provider: str, capabilities: Optional[dict] = None) -> BackendContractDescriptor:
    """The contract a registered device advertised in its capabilities (``backend_contract``), or
    the default one of its provider kind."""
    caps = capabilities or {}
    if isinstance(caps.get("backend_contract"), dict):
        return BackendContractDescriptor.from_json(caps["backend_contract"])
    return BackendContractDescriptor.for_provider(provider if provider in PROVIDERS else "cpu")
