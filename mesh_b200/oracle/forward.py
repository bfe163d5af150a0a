"""fp32 host forward pass (the oracle).

Restates the reference ``LocalForwardPass`` (``agent/src/inference/forward_pass.rs:2988-3147``):
embedding → per layer [RMSNorm → q/k/v → RoPE → KV append (sliding window) → causal attention
with prefix → o_proj → residual → RMSNorm → silu(gate)·up → down → residual] → final RMSNorm →
lm_head on the last row. Weights use the reference's ``[in, out]`` layout. The KV window
(default 4096, ``forward_pass.rs:1795``) trims the oldest rows before an append so that cache plus
incoming rows fit (``forward_pass.rs:1447-1453``).

``LocalForwardPass(weights, shards=n)`` computes the same thing as ``n`` tensor-parallel ranks
whose partial o_proj / down outputs are summed, i.e. the TP algebra with an exact all-reduce.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional

import numpy as np

from ..config import ModelConfig
from ..models.sharding import shard_layout
from .tensor_ops import F32, apply_rope, embed_tokens, matmul, rms_norm, sample_greedy, sample_token, silu


@dataclass
class OracleWeights:
    """Full (unsharded) weights in reference layout: x @ W with W of shape [in, out]."""
    config: ModelConfig
    embedding: np.ndarray
    final_norm: np.ndarray
    lm_head: np.ndarray
    layers: List[Dict[str, np.ndarray]] = field(default_factory=list)

    @classmethod
    def random(cls, cfg: ModelConfig, seed: int = 0, std: float = 0.02) -> "OracleWeights":
        from ..models.weights import synthetic_reference_weights
        return synthetic_reference_weights(cfg, seed=seed, std=std)


def causal_attention_with_prefix(q, k, v, scale, prefix_len):
    t = q.shape[0]
    out = np.zeros((t, v.shape[1]), dtype=F32)
    for r in range(t):
        mk = prefix_len + r + 1
        s = (k[:mk] @ q[r]).astype(F32) * F32(scale)
        s = np.exp(s - s.max()).astype(F32)
        w = s / s.sum(dtype=F32)
        out[r] = (w[:, None] * v[:mk]).sum(0, dtype=F32)
    return out


class LocalForwardPass:
    def __init__(self, weights: OracleWeights, max_seq_len: int = 4096, shards: int = 1):
        self.w = weights
        self.cfg = weights.config
        self.window = max(1, max_seq_len)
        self.shards = shards
        self.k_cache: List[Optional[np.ndarray]] = [None] * self.cfg.num_layers
        self.v_cache: List[Optional[np.ndarray]] = [None] * self.cfg.num_layers
        self.base_position = 0
        self.position = 0

    def clear(self):
        self.k_cache = [None] * self.cfg.num_layers
        self.v_cache = [None] * self.cfg.num_layers
        self.base_position = 0
        self.position = 0

    # -- attention with per-layer sliding window --------------------------------------------
    def _attention(self, layer, positions, q, k, v):
        cfg = self.cfg
        d = cfg.head_dim
        kc, vc = self.k_cache[layer], self.v_cache[layer]
        cur = 0 if kc is None else kc.shape[0]
        inc = len(positions)
        if cur + inc > self.window:
            drop = cur + inc - self.window
            keep = max(cur - drop, 0)
            kc = kc[cur - keep:] if kc is not None else None
            vc = vc[cur - keep:] if vc is not None else None
            if layer == 0:
                self.base_position += cur - keep
        prefix = 0 if kc is None else kc.shape[0]
        qr = apply_rope(q, positions, d, cfg.rope_base)
        kr = apply_rope(k, positions, d, cfg.rope_base)
        kc = kr if kc is None else np.concatenate([kc, kr])
        vc = v.astype(F32) if vc is None else np.concatenate([vc, v.astype(F32)])
        self.k_cache[layer], self.v_cache[layer] = kc, vc
        g = cfg.q_heads_per_kv_head
        scale = 1.0 / np.sqrt(F32(d))
        heads = []
        for h in range(q.shape[1] // d):
            kvh = h // g
            heads.append(causal_attention_with_prefix(
                qr[:, h * d:(h + 1) * d], kc[:, kvh * d:(kvh + 1) * d], vc[:, kvh * d:(kvh + 1) * d], scale, prefix))
        return np.concatenate(heads, 1)

    def _layer(self, li, hidden, positions):
        cfg, L = self.cfg, self.w.layers[li]
        normed = rms_norm(hidden, L["attn_norm"], cfg.rms_norm_eps)
        q, k, v = matmul(normed, L["w_q"]), matmul(normed, L["w_k"]), matmul(normed, L["w_v"])
        attn = self._attention(li, positions, q, k, v)
        if self.shards == 1:
            o = matmul(attn, L["w_o"])
        else:  # sum of per-rank partials (exact all-reduce)
            o = np.zeros_like(hidden, dtype=F32)
            for r in range(self.shards):
                s = shard_layout(cfg, r, self.shards)
                o = o + matmul(attn[:, s.q_start:s.q_start + s.q_cols], L["w_o"][s.q_start:s.q_start + s.q_cols])
        post = (hidden + o).astype(F32)
        mn = rms_norm(post, L["mlp_norm"], cfg.rms_norm_eps)
        act = (silu(matmul(mn, L["w_gate"])) * matmul(mn, L["w_up"])).astype(F32)
        if self.shards == 1:
            down = matmul(act, L["w_down"])
        else:
            down = np.zeros_like(hidden, dtype=F32)
            for r in range(self.shards):
                s = shard_layout(cfg, r, self.shards)
                sl = slice(s.mlp_start, s.mlp_start + s.mlp_cols)
                down = down + matmul(act[:, sl], L["w_down"][sl])
        return (post + down).astype(F32)

    def forward_tokens(self, tokens, start):
        if len(tokens) == 0:
            raise ValueError("Forward pass requires at least one token")
        positions = np.arange(start, start + len(tokens))
        h = embed_tokens(self.w.embedding, tokens)
        for li in range(self.cfg.num_layers):
            h = self._layer(li, h, positions)
        return rms_norm(h, self.w.final_norm, self.cfg.rms_norm_eps)

    def logits_last(self, hidden):
        return matmul(hidden[-1:], self.w.lm_head)[0]

    def prefill(self, tokens) -> np.ndarray:
        if len(tokens) == 0:
            raise ValueError("Cannot prefill an empty prompt without an explicit BOS policy")
        self.clear()
        start = max(0, len(tokens) - self.window)
        self.base_position = start
        h = self.forward_tokens(list(tokens)[start:], start)
        self.position = len(tokens)
        return self.logits_last(h)

    def decode_step(self, token: int) -> np.ndarray:
        if self.position == 0:
            raise ValueError("Decode step requested before prompt prefill")
        h = self.forward_tokens([token], self.position)
        self.position += 1
        return self.logits_last(h)

    def generate(self, prompt, max_new_tokens: int, temperature: float = 0.0, top_p: float = 1.0,
                 seed_base: int = 0) -> list:
        """Greedy (temperature<=0) or seeded sampling; seed = seed_base ^ position
        (reference ``coordinator.rs:2236``)."""
        out = []
        logits = self.prefill(prompt)
        for _ in range(max_new_tokens):
            if temperature <= 0.0:
                tok = sample_greedy(logits)
            else:
                tok = sample_token(logits, temperature, top_p, seed_base ^ self.position)
            out.append(tok)
            if len(out) == max_new_tokens:
                break
            logits = self.decode_step(tok)
        return out
