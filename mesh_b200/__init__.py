"""mesh_b200: a Blackwell-native (B200, sm_100a) tensor-parallel LLM serving framework.

Capabilities follow the Mesh ``zip`` engine and its control plane: sessions with separate
prefill and decode phases, a fair decode queue with a microbatch planner, paged KV with
checkpoint-backed handoff, the ``model.json`` + ``shard-<i>-of-<n>`` on-disk format, the
``mesh`` CLI and the control-plane HTTP API. The compute path is PyTorch for plumbing plus
hand-written sm_100a kernels (tcgen05/TMEM GEMMs fed by TMA, paged GQA attention, fused
all-reduce + residual + RMSNorm over NVLink peer memory).
"""

__version__ = "0.1.0"

from .config import ModelConfig, EngineConfig, PRESETS, get_preset  # noqa: F401
