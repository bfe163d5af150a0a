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
