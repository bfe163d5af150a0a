"""Tensor-parallel fp32 forward pass of one CPU rank (the reference's distributed ForwardPass on
the cpu provider, ``agent/src/inference/forward_pass.rs:1946-2025``): the rank holds its GQA-aligned
q/k/v/o columns and its MLP slice in reference layout; the partial o_proj and down outputs are
summed over the ring (``WorkerRing.all_reduce``); embedding, norms and the LM head are replicated
and the logits are computed from the last row on every rank.
"""
from __future__ import annotations

from typing import Dict, List, Optional

import numpy as np

from ..config import ModelConfig
from ..models.sharding import ShardLayout
from .forward import causal_attention_with_prefix
from .tensor_ops import F32, apply_rope, embed_tokens, matmul, rms_norm, sample_greedy, sample_token, silu


class ShardedForwardPass:
    def __init__(self, cfg: ModelConfig, layout: ShardLayout, tensors: Dict[str, np.ndarray], ring=None,
                 max_seq_len: int = 4096):
        self.cfg = cfg
        self.s = layout
        self.t = tensors
        self.ring = ring
        self.window = max_seq_len
        self.k: List[Optional[np.ndarray]] = [None] * cfg.num_layers
        self.v: List[Optional[np.ndarray]] = [None] * cfg.num_layers
        self.position = 0
        self.allreduce_calls = 0

    def _reduce(self, x: np.ndarray, layer: int) -> np.ndarray:
        self.allreduce_calls += 1
        return x if self.ring is None else self.ring.all_reduce(x, layer=layer)

    def _layer(self, li: int, h: np.ndarray, positions) -> np.ndarray:
        c, t, p = self.cfg, self.t, f"layers.{li}."
        d = c.head_dim
        n = rms_norm(h, t[p + "attn_norm"], c.rms_norm_eps)
        q = apply_rope(matmul(n, t[p + "w_q"]), positions, d, c.rope_base)
        k = apply_rope(matmul(n, t[p + "w_k"]), positions, d, c.rope_base)
        v = matmul(n, t[p + "w_v"])
        kc, vc = self.k[li], self.v[li]
        cur = 0 if kc is None else kc.shape[0]
        if cur + len(positions) > self.window:
            keep = max(cur - (cur + len(positions) - self.window), 0)
            kc, vc = kc[cur - keep:], vc[cur - keep:]
        prefix = 0 if kc is None else kc.shape[0]
        kc = k if kc is None else np.concatenate([kc, k])
        vc = v if vc is None else np.concatenate([vc, v])
        self.k[li], self.v[li] = kc, vc
        g = c.q_heads_per_kv_head
        heads = []
        for hh in range(self.s.local_q_heads):
            kv = hh // g
            heads.append(causal_attention_with_prefix(q[:, hh * d:(hh + 1) * d], kc[:, kv * d:(kv + 1) * d],
                                                      vc[:, kv * d:(kv + 1) * d], 1.0 / np.sqrt(F32(d)), prefix))
        attn = np.concatenate(heads, 1)
        post = (h + self._reduce(matmul(attn, t[p + "w_o"]), 2 * li)).astype(F32)
        m = rms_norm(post, t[p + "mlp_norm"], c.rms_norm_eps)
        act = (silu(matmul(m, t[p + "w_gate"])) * matmul(m, t[p + "w_up"])).astype(F32)
        return (post + self._reduce(matmul(act, t[p + "w_down"]), 2 * li + 1)).astype(F32)

    def _forward(self, tokens, start):
        positions = np.arange(start, start + len(tokens))
        h = embed_tokens(self.t["embedding"], tokens)
        for li in range(self.cfg.num_layers):
            h = self._layer(li, h, positions)
        h = rms_norm(h, self.t["final_norm"], self.cfg.rms_norm_eps)
        return matmul(h[-1:], self.t["lm_head"])[0]

    def prefill(self, tokens) -> np.ndarray:
        self.k = [None] * self.cfg.num_layers
        self.v = [None] * self.cfg.num_layers
        start = max(0, len(tokens) - self.window)
        logits = self._forward(list(tokens)[start:], start)
        self.position = len(tokens)
        return logits

    def decode_step(self, token: int) -> np.ndarray:
        logits = self._forward([token], self.position)
        self.position += 1
        return logits

    def generate(self, prompt, n: int, temperature: float = 0.0, top_p: float = 1.0, seed_base: int = 0):
        out = []
        logits = self.prefill(prompt)
        for i in range(n):
            tok = sample_greedy(logits) if temperature <= 0 else sample_token(logits, temperature, top_p,
                                                                           seed_base ^ self.position)
            out.append(tok)
            if i + 1 < n:
                logits = self.decode_step(tok)
        return out


def shard_reference_weights(w, layout: ShardLayout) -> Dict[str, np.ndarray]:
    """Slice full reference-layout weights (``OracleWeights``) to one rank's shard tensors."""
    s = layout
    t = {"embedding": w.embedding, "final_norm": w.final_norm, "lm_head": w.lm_head}
    ms = slice(s.mlp_start, s.mlp_start + s.mlp_cols)
    for li, L in enumerate(w.layers):
        p = f"layers.{li}."
        t[p + "w_q"] = L["w_q"][:, s.q_start:s.q_start + s.q_cols]
        t[p + "w_k"] = L["w_k"][:, s.kv_start:s.kv_start + s.kv_cols]
        t[p + "w_v"] = L["w_v"][:, s.kv_start:s.kv_start + s.kv_cols]
        t[p + "w_o"] = L["w_o"][s.q_start:s.q_start + s.q_cols]
        t[p + "w_gate"], t[p + "w_up"], t[p + "w_down"] = L["w_gate"][:, ms], L["w_up"][:, ms], L["w_down"][ms]
        t[p + "attn_norm"], t[p + "mlp_norm"] = L["attn_norm"], L["mlp_norm"]
    return t
