"""Model conversion tools: import a Hugging Face Llama checkpoint into the on-disk mesh format, and
re-shard an existing mesh model for another worker count.

    python -m mesh_b200.models.convert hf --src <hf dir> --out <store> --model-id <id> --workers N
    python -m mesh_b200.models.convert reshard --model-dir <store>/<id> --out <store2> --workers M

The reference does the first with ``scripts/fetch_hf_llama_to_meshnet.py:162-368`` (download from
the hub, rename tensors, transpose to ``[in, out]``, write GQA-aligned shards) and the second with
``scripts/reshard_meshnet_model.py:13-120``. Here the checkpoint is read from a local directory
(``config.json`` plus ``*.safetensors`` or ``pytorch_model*.bin``); there is no network access.
Both produce exactly what ``artifacts.write_model`` writes, so ``artifacts.load_shard`` verifies and
loads the result (hashes, shapes, ``mesh.*`` metadata), and the tokenizer files, when present, are
copied next to ``model.json``.
"""
from __future__ import annotations

import argparse
import json
import shutil
from pathlib import Path
from typing import Dict

import numpy as np

from ..config import ModelConfig
from .artifacts import load_model_manifest, load_shard, assignment_for, write_model

TOKENIZER_FILES = ("tokenizer.json", "tokenizer_config.json", "tokenizer.model", "special_tokens_map.json")


def _hf_config(src: Path, name: str) -> ModelConfig:
    c = json.loads((src / "config.json").read_text())
    H = int(c["hidden_size"])
    heads = int(c["num_attention_heads"])
    cfg = ModelConfig(hidden_dim=H, num_heads=heads, num_kv_heads=int(c.get("num_key_value_heads", heads)),
                      num_layers=int(c["num_hidden_layers"]), vocab_size=int(c["vocab_size"]),
                      intermediate_size=int(c["intermediate_size"]), rms_norm_eps=float(c.get("rms_norm_eps", 1e-5)),
                      rope_base=float(c.get("rope_theta", 10000.0)), name=name)
    hd = c.get("head_dim")
    if hd is not None and int(hd) != H // heads:
        raise ValueError(f"head_dim {hd} != hidden_size / num_attention_heads ({H // heads}) is not supported")
    cfg.validate()
    return cfg


def _hf_tensors(src: Path) -> Dict[str, np.ndarray]:
    """Every tensor of the checkpoint as fp32 numpy."""
    out: Dict[str, np.ndarray] = {}
    st = sorted(src.glob("*.safetensors"))
    if st:
        import torch
        from safetensors.torch import load_file
        for f in st:
            for k, v in load_file(str(f)).items():
                out[k] = v.to(torch.float32).numpy()
        return out
    bins = sorted(src.glob("pytorch_model*.bin"))
    if not bins:
        raise FileNotFoundError(f"no *.safetensors or pytorch_model*.bin in {src}")
    import torch
    for f in bins:
        for k, v in torch.load(str(f), map_location="cpu", weights_only=True).items():
            out[k] = v.to(torch.float32).numpy()
    return out


def hf_to_oracle(src: Path, name: str):
    """Read a Hugging Face Llama checkpoint into full reference-layout weights ([in, out] fp32).
    Linear weights are [out, in] in the checkpoint and are transposed; a missing ``lm_head`` (tied
    embeddings) takes the embedding's transpose."""
    from ..oracle.forward import OracleWeights
    src = Path(src)
    cfg = _hf_config(src, name)
    t = _hf_tensors(src)
    pre = "model."

    def get(k):
        if k not in t:
            raise KeyError(f"checkpoint has no tensor {k}")
        return t[k]

    layers = []
    for i in range(cfg.num_layers):
        p = f"{pre}layers.{i}."
        layers.append(dict(
            w_q=get(p + "self_attn.q_proj.weight").T.copy(), w_k=get(p + "self_attn.k_proj.weight").T.copy(),
            w_v=get(p + "self_attn.v_proj.weight").T.copy(), w_o=get(p + "self_attn.o_proj.weight").T.copy(),
            w_up=get(p + "mlp.up_proj.weight").T.copy(), w_gate=get(p + "mlp.gate_proj.weight").T.copy(),
            w_down=get(p + "mlp.down_proj.weight").T.copy(),
            attn_norm=get(p + "input_layernorm.weight").copy(),
            mlp_norm=get(p + "post_attention_layernorm.weight").copy()))
    emb = get(pre + "embed_tokens.weight")
    head = t["lm_head.weight"].T.copy() if "lm_head.weight" in t else emb.T.copy()
    return OracleWeights(config=cfg, embedding=emb.copy(), final_norm=get(pre + "norm.weight").copy(),
                         lm_head=head, layers=layers)


def _copy_tokenizer(src: Path, out: Path):
    for f in TOKENIZER_FILES:
        if (src / f).exists():
            shutil.copyfile(src / f, out / f)


def import_hf_llama(src, out_root, model_id: str, workers: int) -> Path:
    """Hugging Face Llama directory -> ``<out_root>/<model_id>`` with ``workers`` shards."""
    w = hf_to_oracle(Path(src), model_id)
    out = write_model(Path(out_root), model_id, w, workers)
    _copy_tokenizer(Path(src), out)
    return out


def load_full_model(model_dir):
    """Every shard of an on-disk mesh model (hashes and shapes verified), reassembled into full
    reference-layout weights: attention columns and MLP columns concatenated in shard order."""
    from ..oracle.forward import OracleWeights
    model_dir = Path(model_dir)
    man = load_model_manifest(model_dir)
    total = len(list(model_dir.glob("shard-*-of-*.manifest.json")))
    if total == 0:
        raise FileNotFoundError(f"no shard manifests in {model_dir}")
    shards = []
    cfg = None
    for pos in range(total):
        a = assignment_for(model_dir, man["model_id"], pos, total)
        cfg, t = load_shard(model_dir, a)
        shards.append(t)
    cat = lambda key, axis: np.concatenate([s[key] for s in shards], axis=axis)
    layers = []
    for li in range(cfg.num_layers):
        p = f"layers.{li}."
        layers.append(dict(
            w_q=cat(p + "w_q", 1), w_k=cat(p + "w_k", 1), w_v=cat(p + "w_v", 1), w_o=cat(p + "w_o", 0),
            w_up=cat(p + "w_up", 1), w_gate=cat(p + "w_gate", 1), w_down=cat(p + "w_down", 0),
            attn_norm=shards[0][p + "attn_norm"], mlp_norm=shards[0][p + "mlp_norm"]))
    s0 = shards[0]
    return man, OracleWeights(config=cfg, embedding=s0["embedding"], final_norm=s0["final_norm"],
                              lm_head=s0["lm_head"], layers=layers)


def reshard(model_dir, out_root, workers: int) -> Path:
    """Rewrite an on-disk mesh model for ``workers`` shards under ``<out_root>/<model_id>`` (the
    ``execution_layout`` of ``model.json`` and the tokenizer files are kept)."""
    man, w = load_full_model(model_dir)
    out = write_model(Path(out_root), man["model_id"], w, workers, execution_layout=man.get("execution_layout"))
    _copy_tokenizer(Path(model_dir), out)
    return out


def main(argv=None):
    ap = argparse.ArgumentParser(prog="python -m mesh_b200.models.convert")
    sub = ap.add_subparsers(dest="cmd", required=True)
    h = sub.add_parser("hf", help="import a local Hugging Face Llama checkpoint")
    h.add_argument("--src", required=True)
    h.add_argument("--out", required=True)
    h.add_argument("--model-id", required=True)
    h.add_argument("--workers", type=int, default=1)
    r = sub.add_parser("reshard", help="rewrite an on-disk mesh model for another worker count")
    r.add_argument("--model-dir", required=True)
    r.add_argument("--out", required=True)
    r.add_argument("--workers", type=int, required=True)
    a = ap.parse_args(argv)
    if a.cmd == "hf":
        out = import_hf_llama(a.src, a.out, a.model_id, a.workers)
    else:
        out = reshard(a.model_dir, a.out, a.workers)
    print(json.dumps({"model_dir": str(out)}))


if __name__ == "__main__":
    main()
