"""Sharding rules, weight layouts and the on-disk artifact format (CPU)."""
import json

import numpy as np
import pytest
import torch

from mesh_b200.config import ModelConfig, get_preset
from mesh_b200.models import artifacts
from mesh_b200.models.sharding import even_split, shard_layout, validate_column_range
from mesh_b200.models.weights import (GU_BLOCK, deinterleave_gate_up, device_weights_from_reference,
                                      interleave_gate_up, synthetic_reference_weights)


def test_even_split_matches_reference_partition():
    # remainder to the lowest positions (scripts/fetch_hf_llama_to_meshnet.py:22-40)
    assert [even_split(10, 3, i) for i in range(3)] == [(0, 4), (4, 3), (7, 3)]
    assert sum(even_split(14336, 8, i)[1] for i in range(8)) == 14336


@pytest.mark.parametrize("name,world", [("llama3-8b", 8), ("llama3-70b", 8), ("tinyllama-1.1b", 2), ("llama3-8b", 3)])
def test_shard_layout_gqa_aligned(name, world):
    cfg = get_preset(name)
    covered_q, covered_kv, covered_mlp = 0, 0, 0
    for r in range(world):
        s = shard_layout(cfg, r, world)
        assert s.q_start % cfg.q_group_width == 0 and s.q_cols % cfg.q_group_width == 0
        assert s.local_q_heads == s.local_kv_heads * cfg.q_heads_per_kv_head
        assert s.q_start == covered_q and s.kv_start == covered_kv and s.mlp_start == covered_mlp
        covered_q += s.q_cols
        covered_kv += s.kv_cols
        covered_mlp += s.mlp_cols
        validate_column_range(cfg, s.column_start, s.column_end)
    assert covered_q == cfg.hidden_dim and covered_kv == cfg.kv_dim and covered_mlp == cfg.intermediate_size


def test_shard_layout_rejects_too_many_ranks_and_misaligned():
    cfg = get_preset("llama3-8b")
    with pytest.raises(ValueError):
        shard_layout(cfg, 0, 16)
    with pytest.raises(ValueError):
        validate_column_range(cfg, 0, 100)


def test_gate_up_interleave_roundtrip():
    g = torch.randn(192, 16)
    u = torch.randn(192, 16)
    x = interleave_gate_up(g, u, 192)
    assert torch.equal(x[:GU_BLOCK], g[:GU_BLOCK]) and torch.equal(x[GU_BLOCK:2 * GU_BLOCK], u[:GU_BLOCK])
    g2, u2 = deinterleave_gate_up(x)
    assert torch.equal(g2, g) and torch.equal(u2, u)


def test_device_weights_are_transposed_slices():
    cfg = get_preset("tiny")
    w = synthetic_reference_weights(cfg, seed=1)
    d = device_weights_from_reference(w, 1, 2, dtype=torch.float32)
    s = shard_layout(cfg, 1, 2)
    L = w.layers[0]
    assert torch.allclose(d.layers[0].wqkv[:s.q_cols], torch.from_numpy(L["w_q"][:, s.q_start:s.q_start + s.q_cols].T))
    assert torch.allclose(d.layers[0].wo, torch.from_numpy(L["w_o"][s.q_start:s.q_start + s.q_cols].T))
    g, u = deinterleave_gate_up(d.layers[0].wgu)
    ms = slice(s.mlp_start, s.mlp_start + s.mlp_cols)
    assert torch.allclose(g[:s.mlp_cols], torch.from_numpy(L["w_gate"][:, ms].T))
    assert d.lm_head.shape == (d.vocab_local, cfg.hidden_dim)


def test_artifacts_roundtrip_and_validation(tmp_path):
    cfg = get_preset("tiny")
    w = synthetic_reference_weights(cfg, seed=2)
    out = artifacts.write_model(tmp_path, "tiny-model", w, workers=2)
    man = json.loads((out / "model.json").read_text())
    assert man["tensor_parallelism_dim"] == cfg.hidden_dim and man["kv_head_count"] == cfg.num_kv_heads
    a = artifacts.assignment_for(out, "tiny-model", 1, 2)
    cfg2, t = artifacts.load_shard(out, a)
    assert cfg2.hidden_dim == cfg.hidden_dim and cfg2.rope_base == cfg.rope_base
    s = shard_layout(cfg, 1, 2)
    np.testing.assert_array_equal(t["layers.0.w_q"], w.layers[0]["w_q"][:, s.q_start:s.q_start + s.q_cols])
    dw = artifacts.shard_to_device_weights(cfg2, t, 1, 2)
    assert dw.layers[0].wqkv.shape == (s.q_cols + 2 * s.kv_cols, cfg.hidden_dim)
    # a wrong assignment and a corrupted file are both rejected
    with pytest.raises(artifacts.ArtifactError):
        artifacts.load_shard(out, artifacts.ShardAssignment("tiny-model", 1, 2, 0, s.column_end))
    p = out / "shard-1-of-2.safetensors"
    b = bytearray(p.read_bytes())
    b[-1] ^= 0xFF
    p.write_bytes(bytes(b))
    with pytest.raises(artifacts.ArtifactError):
        artifacts.load_shard(out, a)


def test_prefill_split_point_and_sub_meta():
    """The overlapped-prefill split: the prompt boundary nearest half the tokens with both halves of
    at least 512 tokens, and sub-steps whose rows, tables and offsets are rebased."""
    import types
    import torch
    from mesh_b200.models.llama import LlamaRunner, StepMeta
    cu = [0, 300, 580, 890, 1180, 1310]
    T, S = cu[-1], len(cu) - 1
    m = StepMeta(ids=torch.arange(T, dtype=torch.int32), pos=torch.arange(T, dtype=torch.int32),
                 slot=torch.arange(T, dtype=torch.int64), block_tables=torch.arange(S * 4, dtype=torch.int32).view(S, 4),
                 seq_lens=torch.tensor([cu[i + 1] - cu[i] for i in range(S)], dtype=torch.int32),
                 cu_q=torch.tensor(cu, dtype=torch.int32), last_idx=torch.tensor(cu[1:], dtype=torch.int64) - 1,
                 max_q_len=310, decode=False, cu_host=cu)
    on = types.SimpleNamespace(overlap_prefill=True)
    assert LlamaRunner._split_point(on, m) == 2
    assert LlamaRunner._split_point(types.SimpleNamespace(overlap_prefill=False), m) == 0
    small = StepMeta(ids=m.ids[:600], pos=m.pos, slot=m.slot, block_tables=m.block_tables, seq_lens=m.seq_lens,
                     decode=False, cu_host=[0, 300, 600])
    assert LlamaRunner._split_point(on, small) == 0  # halves under 512 tokens
    a, b = LlamaRunner._sub_meta(m, 0, 2), LlamaRunner._sub_meta(m, 2, S)
    assert a.ids.shape[0] == 580 and b.ids.shape[0] == 730 and int(b.ids[0]) == 580
    assert b.cu_q.tolist() == [0, 310, 600, 730] and b.cu_host == [0, 310, 600, 730]
    assert b.last_idx.tolist() == [309, 599, 729] and a.last_idx.tolist() == [299, 579]
    assert b.block_tables.tolist() == m.block_tables[2:].tolist() and b.max_q_len == 310 and a.max_q_len == 300
    assert not a.decode and not b.decode
