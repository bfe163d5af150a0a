"""CPU oracle: hand-computed cases (ported from the reference's tensor_ops tests) and torch fp32."""
import numpy as np
import pytest
import torch

from mesh_b200.config import get_preset
from mesh_b200.oracle import tensor_ops as T
from mesh_b200.oracle.forward import LocalForwardPass
from mesh_b200.models.weights import synthetic_reference_weights


def test_matmul_hand():
    a = np.array([[1, 2], [3, 4]], np.float32)
    b = np.array([[5, 6], [7, 8]], np.float32)
    assert T.matmul(a, b).tolist() == [[19, 22], [43, 50]]
    with pytest.raises(ValueError):
        T.matmul(a, np.ones((3, 1), np.float32))


def test_silu_gelu_softmax_rms():
    x = np.array([[0.0, 1.0, -1.0]], np.float32)
    np.testing.assert_allclose(T.silu(x), x / (1 + np.exp(-x)), rtol=1e-6)
    s = T.softmax(np.array([[1.0, 2.0, 3.0]], np.float32))
    np.testing.assert_allclose(s.sum(), 1.0, rtol=1e-6)
    assert s[0, 2] > s[0, 1] > s[0, 0]
    r = T.rms_norm(np.array([[3.0, 4.0]], np.float32), np.ones(2, np.float32), 0.0)
    np.testing.assert_allclose(r, [[3 / np.sqrt(12.5), 4 / np.sqrt(12.5)]], rtol=1e-6)
    g = T.gelu(np.array([0.0], np.float32))
    assert g[0] == 0.0


def test_rope_position_zero_identity_and_norm_preserved():
    x = np.random.default_rng(0).standard_normal((3, 8)).astype(np.float32)
    out = T.apply_rope(x, [0, 5, 100], 4, 10000.0)
    np.testing.assert_allclose(out[0], x[0], rtol=1e-6)
    for r in range(3):
        for h in range(2):
            a = x[r, h * 4:(h + 1) * 4]
            b = out[r, h * 4:(h + 1) * 4]
            np.testing.assert_allclose(np.linalg.norm(a), np.linalg.norm(b), rtol=1e-5)
    with pytest.raises(ValueError):
        T.apply_rope(x, [0, 1], 4, 1e4)


def test_sampling_threshold_and_greedy():
    t = T.deterministic_sample_threshold(0)
    assert 0.0 <= t < 1.0
    assert T.deterministic_sample_threshold(0) == t  # deterministic
    assert len({T.deterministic_sample_threshold(s) for s in range(100)}) > 90
    logits = np.array([0.1, 3.0, 3.0, -1.0], np.float32)
    assert T.sample_greedy(logits) == 1  # first maximal index


def test_sample_token_host_vs_device_semantics_agree():
    rng = np.random.default_rng(5)
    for trial in range(50):
        logits = rng.standard_normal(64).astype(np.float32) * 3
        for temp, top_p in [(1.0, 1.0), (0.7, 0.9), (1.3, 0.5)]:
            seed = trial * 7 + 3
            h = T.sample_token(logits, temp, top_p, seed)
            d = T.sample_tokens_device_semantics(logits[None], temp, top_p, [seed])[0]
            assert h == d


def test_sample_token_extreme_top_p_picks_argmax():
    logits = np.array([1.0, 5.0, 2.0], np.float32)
    assert T.sample_token(logits, 1.0, 1e-6, 11) == 1


def test_embed_bounds():
    table = np.arange(12, dtype=np.float32).reshape(4, 3)
    assert T.embed_tokens(table, [2, 0]).tolist() == [[6, 7, 8], [0, 1, 2]]
    with pytest.raises(ValueError):
        T.embed_tokens(table, [4])


def test_oracle_matches_torch_fp32_reference():
    cfg = get_preset("tiny")
    w = synthetic_reference_weights(cfg, seed=2)
    prompt = [1, 5, 9, 100, 7, 300]
    orc = LocalForwardPass(w)
    logits = orc.prefill(prompt)
    # independent torch restatement
    H, D = cfg.hidden_dim, cfg.head_dim
    x = torch.from_numpy(w.embedding[prompt])
    pos = torch.arange(len(prompt), dtype=torch.float64)
    half = D // 2
    inv = 1.0 / (cfg.rope_base ** (torch.arange(half, dtype=torch.float64) * 2 / D))
    ang = pos[:, None] * inv[None]
    cos, sin = torch.cos(ang).float(), torch.sin(ang).float()

    def rope(t):
        t = t.view(len(prompt), -1, D)
        l, r = t[..., :half], t[..., half:]
        return torch.cat([l * cos[:, None] - r * sin[:, None], l * sin[:, None] + r * cos[:, None]], -1)

    def rms(t, g):
        return t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + cfg.rms_norm_eps) * torch.from_numpy(g)

    for L in w.layers:
        n = rms(x, L["attn_norm"])
        q = rope(n @ torch.from_numpy(L["w_q"]))
        k = rope(n @ torch.from_numpy(L["w_k"]))
        v = (n @ torch.from_numpy(L["w_v"])).view(len(prompt), -1, D)
        g = cfg.q_heads_per_kv_head
        k = k.repeat_interleave(g, 1)
        v = v.repeat_interleave(g, 1)
        s = torch.einsum("qhd,khd->hqk", q, k) / np.sqrt(D)
        s = s.masked_fill(torch.triu(torch.ones(len(prompt), len(prompt), dtype=torch.bool), 1), float("-inf"))
        a = torch.einsum("hqk,khd->qhd", torch.softmax(s, -1), v).reshape(len(prompt), -1)
        x = x + a @ torch.from_numpy(L["w_o"])
        n = rms(x, L["mlp_norm"])
        x = x + (torch.nn.functional.silu(n @ torch.from_numpy(L["w_gate"])) * (n @ torch.from_numpy(L["w_up"]))) @ \
            torch.from_numpy(L["w_down"])
    x = rms(x, w.final_norm)
    want = (x[-1] @ torch.from_numpy(w.lm_head)).numpy()
    np.testing.assert_allclose(logits, want, rtol=2e-3, atol=2e-4)


def test_incremental_decode_equals_full_recompute():
    """reference forward_pass.rs:3270-3292: decode with cache == prefill of the longer prompt."""
    cfg = get_preset("tiny")
    w = synthetic_reference_weights(cfg, seed=4)
    prompt = [3, 4, 5, 6]
    a = LocalForwardPass(w)
    a.prefill(prompt)
    inc = a.decode_step(42)
    full = LocalForwardPass(w).prefill(prompt + [42])
    np.testing.assert_allclose(inc, full, rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("shards", [2])
def test_tp_partial_sums_equal_full(shards):
    cfg = get_preset("tiny")
    w = synthetic_reference_weights(cfg, seed=6)
    p = [9, 8, 7, 6, 5]
    np.testing.assert_allclose(LocalForwardPass(w, shards=shards).prefill(p), LocalForwardPass(w).prefill(p),
                               rtol=1e-4, atol=1e-5)


def test_sliding_window_trims_oldest():
    cfg = get_preset("tiny")
    w = synthetic_reference_weights(cfg, seed=8)
    f = LocalForwardPass(w, max_seq_len=4)
    f.prefill([1, 2, 3, 4, 5, 6])
    assert f.base_position == 2
    assert f.k_cache[0].shape[0] == 4
    f.decode_step(7)
    assert f.k_cache[0].shape[0] == 4


def test_torch_sampler_matches_device_semantics_oracle():
    import torch
    from mesh_b200.ops.sampling import sample
    rng = np.random.default_rng(9)
    for trial in range(40):
        logits = (rng.standard_normal((3, 50)) * 2.5).astype(np.float32)
        seeds = [trial * 31 + i for i in range(3)]
        for temp, top_p in [(1.0, 1.0), (0.7, 0.9), (1.3, 0.3), (0.0, 0.9)]:
            got = sample(torch.from_numpy(logits), temp, top_p, seeds).tolist()
            want = T.sample_tokens_device_semantics(logits, temp, top_p, seeds)
            assert got == want, (trial, temp, top_p)
