"""On-disk model format: ``model.json`` plus ``shard-<i>-of-<n>.{manifest.json,safetensors}``.

Compatible with the reference layout (``README.md:195-206``; writer
``scripts/fetch_hf_llama_to_meshnet.py:162-368``; reader ``agent/src/inference/artifact_loader.rs``):

* ``model.json``: model_id, tensor_parallelism_dim, attention_head_count, kv_head_count,
  total_model_bytes, tokenizer_file, tokenizer_config_file (+ optional execution_layout);
* each shard holds ``embedding``, ``final_norm``, ``lm_head`` (replicated) and
  ``layers.<i>.{w_q,w_k,w_v,w_o,w_up,w_gate,w_down,attn_norm,mlp_norm}`` in ``[in, out]`` layout;
* safetensors metadata carries ``mesh.*`` model geometry plus the shard assignment;
* the manifest records the assignment and the file's SHA-256, verified on load.

Tensors are F32 as in the reference; bf16 files are accepted as an extension (``dtype="bf16"``).
"""
from __future__ import annotations

import hashlib
import json
import os
from dataclasses import dataclass
from pathlib import Path
from typing import Dict, Optional

import numpy as np

from ..config import ModelConfig
from .sharding import shard_layout, validate_column_range

LAYER_KEYS = ("w_q", "w_k", "w_v", "w_o", "w_up", "w_gate", "w_down", "attn_norm", "mlp_norm")


def model_store_dir() -> Path:
    env = os.environ.get("MESHNET_MODEL_STORE")
    if env:
        return Path(env)
    home = os.environ.get("MESHNET_HOME")
    return (Path(home) if home else Path.home() / ".meshnet") / "models"


def _save_json(path: Path, payload: dict) -> None:
    path.write_text(json.dumps(payload, indent=2, sort_keys=True) + "\n", encoding="utf-8")


def sha256_file(path: Path) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 22), b""):
            h.update(chunk)
    return h.hexdigest()


def write_model(out_root: Path, model_id: str, weights, workers: int, dtype: str = "f32",
                execution_layout: Optional[dict] = None) -> Path:
    """Write ``weights`` (``OracleWeights``) as ``workers`` GQA-aligned shards."""
    from safetensors.numpy import save_file
    cfg: ModelConfig = weights.config
    out = Path(out_root) / model_id
    out.mkdir(parents=True, exist_ok=True)
    np_dtype = np.float32
    manifest = {
        "model_id": model_id,
        "tensor_parallelism_dim": cfg.hidden_dim,
        "attention_head_count": cfg.num_heads,
        "kv_head_count": cfg.num_kv_heads,
        "total_model_bytes": int(cfg.param_count() * 4),
        "tokenizer_file": "tokenizer.json",
        "tokenizer_config_file": "tokenizer_config.json",
        "num_layers": cfg.num_layers,
    }
    if execution_layout:
        manifest["execution_layout"] = execution_layout
    _save_json(out / "model.json", manifest)
    base_md = cfg.to_metadata(model_id)
    for pos in range(workers):
        s = shard_layout(cfg, pos, workers)
        tensors: Dict[str, np.ndarray] = {
            "embedding": weights.embedding, "final_norm": weights.final_norm, "lm_head": weights.lm_head,
        }
        ms = slice(s.mlp_start, s.mlp_start + s.mlp_cols)
        for li, L in enumerate(weights.layers):
            tensors[f"layers.{li}.w_q"] = L["w_q"][:, s.q_start:s.q_start + s.q_cols]
            tensors[f"layers.{li}.w_k"] = L["w_k"][:, s.kv_start:s.kv_start + s.kv_cols]
            tensors[f"layers.{li}.w_v"] = L["w_v"][:, s.kv_start:s.kv_start + s.kv_cols]
            tensors[f"layers.{li}.w_o"] = L["w_o"][s.q_start:s.q_start + s.q_cols]
            tensors[f"layers.{li}.w_up"] = L["w_up"][:, ms]
            tensors[f"layers.{li}.w_gate"] = L["w_gate"][:, ms]
            tensors[f"layers.{li}.w_down"] = L["w_down"][ms]
            tensors[f"layers.{li}.attn_norm"] = L["attn_norm"]
            tensors[f"layers.{li}.mlp_norm"] = L["mlp_norm"]
        tensors = {k: np.ascontiguousarray(v, dtype=np_dtype) for k, v in tensors.items()}
        md = dict(base_md)
        md.update({"mesh.worker_position": str(pos), "mesh.total_workers": str(workers),
                   "mesh.column_start": str(s.column_start), "mesh.column_end": str(s.column_end)})
        path = out / f"shard-{pos}-of-{workers}.safetensors"
        save_file(tensors, str(path), metadata=md)
        _save_json(out / f"shard-{pos}-of-{workers}.manifest.json", {
            "model_id": model_id, "worker_position": pos, "total_workers": workers,
            "column_start": s.column_start, "column_end": s.column_end,
            "expected_sha256": sha256_file(path),
        })
    return out


@dataclass
class ShardAssignment:
    model_id: str
    worker_position: int
    total_workers: int
    column_start: int
    column_end: int


class ArtifactError(ValueError):
    pass


def load_shard(model_dir: Path, assignment: ShardAssignment, verify_hash: bool = True):
    """Load and validate one shard; returns ``(ModelConfig, dict of numpy arrays)``
    (reference ``ArtifactShardLoader``, ``artifact_loader.rs:40-584``)."""
    from safetensors import safe_open
    model_dir = Path(model_dir)
    a = assignment
    mpath = model_dir / f"shard-{a.worker_position}-of-{a.total_workers}.manifest.json"
    wpath = model_dir / f"shard-{a.worker_position}-of-{a.total_workers}.safetensors"
    try:
        man = json.loads(mpath.read_text())
    except FileNotFoundError as e:
        raise ArtifactError(f"Failed to read shard manifest {mpath}: {e}") from e
    if (man["model_id"] != a.model_id or man["worker_position"] != a.worker_position
            or man["total_workers"] != a.total_workers or man["column_start"] != a.column_start
            or man["column_end"] != a.column_end):
        raise ArtifactError(f"Shard manifest does not match requested assignment for model {a.model_id}")
    if verify_hash:
        digest = sha256_file(wpath)
        if digest != man["expected_sha256"]:
            raise ArtifactError(f"Artifact hash mismatch for {wpath}: expected {man['expected_sha256']}, got {digest}")
    with safe_open(str(wpath), framework="np") as f:
        md = f.metadata() or {}
        if not md:
            raise ArtifactError("Safetensors shard missing metadata")
        if md.get("mesh.model_id") != a.model_id:
            raise ArtifactError(f"Safetensors metadata model_id mismatch: expected {a.model_id}, got {md.get('mesh.model_id')}")
        if (int(md["mesh.worker_position"]) != a.worker_position or int(md["mesh.total_workers"]) != a.total_workers):
            raise ArtifactError(f"Safetensors metadata shard assignment mismatch for model {a.model_id}")
        if int(md["mesh.column_start"]) != a.column_start or int(md["mesh.column_end"]) != a.column_end:
            raise ArtifactError(f"Safetensors metadata shard range mismatch for model {a.model_id}")
        cfg = ModelConfig.from_metadata(md)
        tensors = {k: f.get_tensor(k) for k in f.keys()}
    for k, v in tensors.items():
        if v.dtype not in (np.float32,) and str(v.dtype) != "bfloat16":
            raise ArtifactError(f"Tensor {k} must be F32, got {v.dtype}")
    _validate_shapes(cfg, a, tensors)
    return cfg, tensors


def _validate_shapes(cfg: ModelConfig, a: ShardAssignment, t: Dict[str, np.ndarray]) -> None:
    q_cols, kv_cols = validate_column_range(cfg, a.column_start, a.column_end)
    H, V = cfg.hidden_dim, cfg.vocab_size
    from .sharding import even_split
    _, mlp = even_split(cfg.intermediate_size, a.total_workers, a.worker_position)

    def want(name, shape):
        if name not in t:
            raise ArtifactError(f"Missing tensor {name}")
        if tuple(t[name].shape) != tuple(shape):
            raise ArtifactError(f"Tensor {name} shape mismatch: expected {shape}, got {tuple(t[name].shape)}")
    want("embedding", (V, H))
    want("final_norm", (H,))
    want("lm_head", (H, V))
    for li in range(cfg.num_layers):
        p = f"layers.{li}."
        want(p + "w_q", (H, q_cols)); want(p + "w_k", (H, kv_cols)); want(p + "w_v", (H, kv_cols))
        want(p + "w_o", (q_cols, H)); want(p + "w_up", (H, mlp)); want(p + "w_gate", (H, mlp))
        want(p + "w_down", (mlp, H)); want(p + "attn_norm", (H,)); want(p + "mlp_norm", (H,))


def load_model_manifest(model_dir: Path) -> dict:
    return json.loads((Path(model_dir) / "model.json").read_text())


def assignment_for(model_dir: Path, model_id: str, position: int, total: int) -> ShardAssignment:
    man = json.loads((Path(model_dir) / f"shard-{position}-of-{total}.manifest.json").read_text())
    return ShardAssignment(model_id, position, total, man["column_start"], man["column_end"])


def shard_to_device_weights(cfg: ModelConfig, tensors: Dict[str, np.ndarray], rank: int, world: int,
                            device="cpu"):
    """Convert a loaded shard (already this rank's columns) into device layout."""
    import torch
    from .weights import DeviceWeights, LayerDeviceWeights, GU_BLOCK, interleave_gate_up, pad_to
    from .sharding import even_split
    s = shard_layout(cfg, rank, world)
    i_pad = pad_to(s.mlp_cols, GU_BLOCK)
    v0, vn = even_split(cfg.vocab_size, world, rank)

    def d(x):
        return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(device=device, dtype=torch.bfloat16)
    layers = []
    for li in range(cfg.num_layers):
        p = f"layers.{li}."
        wd = tensors[p + "w_down"].T
        if i_pad != s.mlp_cols:
            wd = np.concatenate([wd, np.zeros((wd.shape[0], i_pad - s.mlp_cols), np.float32)], 1)
        layers.append(LayerDeviceWeights(
            wqkv=d(np.concatenate([tensors[p + "w_q"].T, tensors[p + "w_k"].T, tensors[p + "w_v"].T])),
            wo=d(tensors[p + "w_o"].T),
            wgu=interleave_gate_up(d(tensors[p + "w_gate"].T), d(tensors[p + "w_up"].T), i_pad),
            wdown=d(wd), attn_norm=d(tensors[p + "attn_norm"]), mlp_norm=d(tensors[p + "mlp_norm"])))
    return DeviceWeights(config=cfg, layout=s, vocab_start=v0, vocab_local=vn, i_pad=i_pad,
                         embedding=d(tensors["embedding"][v0:v0 + vn]), final_norm=d(tensors["final_norm"]),
                         lm_head=d(tensors["lm_head"][:, v0:v0 + vn].T), layers=layers)
