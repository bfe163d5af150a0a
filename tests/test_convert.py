"""Model conversion: a Hugging Face Llama checkpoint (a tiny random model saved by transformers)
imported into the mesh format gives the same logits in the oracle as transformers' own forward,
and re-sharding 1 -> 2 -> 1 workers gives back the same tensors."""
import json

import numpy as np
import pytest
import torch


def _tiny_hf(path):
    transformers = pytest.importorskip("transformers")
    cfg = transformers.LlamaConfig(hidden_size=128, intermediate_size=320, num_attention_heads=4,
                                   num_key_value_heads=2, num_hidden_layers=2, vocab_size=300,
                                   rms_norm_eps=1e-5, rope_theta=10000.0, tie_word_embeddings=False)
    torch.manual_seed(0)
    model = transformers.LlamaForCausalLM(cfg).eval()
    model.save_pretrained(str(path), safe_serialization=True)
    return model


def test_hf_import_matches_transformers_logits(tmp_path):
    from mesh_b200.models.convert import import_hf_llama, load_full_model
    from mesh_b200.oracle.forward import LocalForwardPass
    model = _tiny_hf(tmp_path / "hf")
    out = import_hf_llama(tmp_path / "hf", tmp_path / "store", "tiny-hf", workers=2)
    assert json.loads((out / "model.json").read_text())["kv_head_count"] == 2
    _, w = load_full_model(out)
    prompt = [5, 17, 250, 3, 99, 42]
    got = np.asarray(LocalForwardPass(w).prefill(prompt), dtype=np.float32)
    with torch.no_grad():
        ref = model(torch.tensor([prompt])).logits[0, -1].float().numpy()
    assert got.shape == ref.shape
    assert np.abs(got - ref).max() < 1e-3 * max(1.0, float(np.abs(ref).max()))


def test_reshard_roundtrip(tmp_path):
    from mesh_b200.config import get_preset
    from mesh_b200.models.artifacts import write_model
    from mesh_b200.models.convert import load_full_model, reshard
    from mesh_b200.models.weights import synthetic_reference_weights
    w = synthetic_reference_weights(get_preset("tiny-gqa"), seed=4)
    src = write_model(tmp_path / "a", "m", w, 1)
    two = reshard(src, tmp_path / "b", 2)
    one = reshard(two, tmp_path / "c", 1)
    assert len(list(two.glob("shard-*-of-2.safetensors"))) == 2
    _, back = load_full_model(one)
    assert np.array_equal(back.embedding, w.embedding) and np.array_equal(back.lm_head, w.lm_head)
    for a, b in zip(back.layers, w.layers):
        for k in a:
            assert np.array_equal(a[k], b[k]), k


def test_mesh_model_cli(tmp_path, monkeypatch, capsys):
    """`mesh model import-hf | info | reshard | list` over the model store and the shard registry."""
    from mesh_b200.cli import main as cli
    monkeypatch.setenv("MESHNET_HOME", str(tmp_path / "home"))
    monkeypatch.setenv("MESHNET_MODEL_STORE", str(tmp_path / "store"))
    _tiny_hf(tmp_path / "hf")
    assert cli.main(["model", "import-hf", "--src", str(tmp_path / "hf"), "--model-id", "tiny-hf", "--workers", "2"]) == 0
    out = json.loads(capsys.readouterr().out)
    assert (tmp_path / "store" / "tiny-hf" / "shard-1-of-2.safetensors").exists() and out["model_dir"]
    assert cli.main(["model", "info", "--model-id", "tiny-hf", "--gpu-bytes", str(10 ** 9)]) == 0
    info = json.loads(capsys.readouterr().out)
    assert info["num_layers"] == 2 and info["num_kv_heads"] == 2 and info["min_workers"] == 1
    assert cli.main(["model", "reshard", "--model-id", "tiny-hf", "--workers", "1"]) == 0
    re_dir = json.loads(capsys.readouterr().out)["model_dir"]
    assert (tmp_path / "store" / "tiny-hf-tp1" / "tiny-hf" / "shard-0-of-1.safetensors").exists(), re_dir
    assert cli.main(["model", "list"]) == 0
    lst = json.loads(capsys.readouterr().out)
    assert "tiny-hf" in lst["models"] and "tiny-hf" in lst["registry"]["models"]
