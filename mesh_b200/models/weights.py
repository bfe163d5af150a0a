"""Synthetic weights and the per-rank device weight layout.

Reference layout (``[in, out]`` fp32, what the artifact files hold) is produced by
``synthetic_reference_weights``. The device layout used by the sm_100a kernels is
``[out, in]`` bf16 (K-major operands for tcgen05), per rank:

* ``wqkv``  [q_cols + 2*kv_cols, H]   rows: local q heads, local k heads, local v heads
* ``wo``    [H, q_cols]
* ``wgu``   [2*I_pad, H]  gate/up rows interleaved in blocks of 64 (g0..63, u0..63, g64..127, ...)
            so one 128-row (or 128-column) GEMM tile holds matching gate and up features and the
            SiLU·up epilogue stays inside the tile; I_pad rounds the local width up to 64 with zeros
* ``wdown`` [H, I_pad]
* ``lm_head`` [V_local, H]  vocab-parallel rows (the reference replicates the full head)
* ``embedding`` [V, H] at TP=1; at TP>1 only this rank's vocabulary rows [vocab_start, +vocab_local)
  (the same split as the LM head; other ranks' rows are read over NVLink); norms [H].
"""
from __future__ import annotations

import hashlib
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import numpy as np
import torch

from ..config import ModelConfig
from .sharding import ShardLayout, even_split, shard_layout

GU_BLOCK = 64


def _seed_for(seed: int, *parts) -> int:
    h = hashlib.sha256(("%d|" % seed + "|".join(str(p) for p in parts)).encode()).digest()
    return int.from_bytes(h[:8], "little") & ((1 << 63) - 1)


def synthetic_reference_weights(cfg: ModelConfig, seed: int = 0, std: float = 0.02):
    """Full fp32 weights in reference layout, N(0, std) from ``seed``; norms are 1 + N(0, std)."""
    from ..oracle.forward import OracleWeights
    cfg.validate()
    rng = np.random.default_rng(seed)
    H, I, V, kv = cfg.hidden_dim, cfg.intermediate_size, cfg.vocab_size, cfg.kv_dim

    def n(*shape):
        return (rng.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float32)

    layers = []
    for _ in range(cfg.num_layers):
        layers.append(dict(
            w_q=n(H, H), w_k=n(H, kv), w_v=n(H, kv), w_o=n(H, H),
            w_up=n(H, I), w_gate=n(H, I), w_down=n(I, H),
            attn_norm=(1.0 + n(H)).astype(np.float32), mlp_norm=(1.0 + n(H)).astype(np.float32),
        ))
    return OracleWeights(config=cfg, embedding=n(V, H), final_norm=(1.0 + n(H)).astype(np.float32),
                         lm_head=n(H, V), layers=layers)


def pad_to(x: int, m: int) -> int:
    return (x + m - 1) // m * m


@dataclass
class LayerDeviceWeights:
    wqkv: torch.Tensor
    wo: torch.Tensor
    wgu: torch.Tensor
    wdown: torch.Tensor
    attn_norm: torch.Tensor
    mlp_norm: torch.Tensor


@dataclass
class DeviceWeights:
    """Per-rank weights in device layout."""
    config: ModelConfig
    layout: ShardLayout
    vocab_start: int
    vocab_local: int
    i_pad: int
    embedding: torch.Tensor
    final_norm: torch.Tensor
    lm_head: torch.Tensor
    layers: List[LayerDeviceWeights] = field(default_factory=list)

    def nbytes(self) -> int:
        t = [self.embedding, self.final_norm, self.lm_head]
        for L in self.layers:
            t += [L.wqkv, L.wo, L.wgu, L.wdown, L.attn_norm, L.mlp_norm]
        return sum(x.numel() * x.element_size() for x in t)


def interleave_gate_up(gate_t: torch.Tensor, up_t: torch.Tensor, i_pad: int) -> torch.Tensor:
    """gate_t/up_t: [I_loc, H] (rows = features). Returns [2*i_pad, H] interleaved by GU_BLOCK."""
    i_loc, h = gate_t.shape
    if i_pad != i_loc:
        z = torch.zeros(i_pad - i_loc, h, dtype=gate_t.dtype, device=gate_t.device)
        gate_t, up_t = torch.cat([gate_t, z]), torch.cat([up_t, z])
    nb = i_pad // GU_BLOCK
    g = gate_t.reshape(nb, GU_BLOCK, h)
    u = up_t.reshape(nb, GU_BLOCK, h)
    return torch.stack([g, u], 1).reshape(2 * i_pad, h).contiguous()


def deinterleave_gate_up(wgu: torch.Tensor):
    two_i, h = wgu.shape
    nb = two_i // (2 * GU_BLOCK)
    x = wgu.reshape(nb, 2, GU_BLOCK, h)
    return x[:, 0].reshape(-1, h), x[:, 1].reshape(-1, h)


def device_weights_from_reference(w, rank: int, world: int, device="cpu", dtype=torch.bfloat16) -> DeviceWeights:
    """Shard full reference-layout weights (``OracleWeights``) for ``rank`` and convert to device layout."""
    cfg = w.config
    s = shard_layout(cfg, rank, world)
    i_pad = pad_to(s.mlp_cols, GU_BLOCK)
    v0, vn = even_split(cfg.vocab_size, world, rank)

    def t(a):
        return torch.from_numpy(np.ascontiguousarray(a)).to(device=device, dtype=dtype)

    layers = []
    for L in w.layers:
        q = L["w_q"][:, s.q_start:s.q_start + s.q_cols].T
        k = L["w_k"][:, s.kv_start:s.kv_start + s.kv_cols].T
        v = L["w_v"][:, s.kv_start:s.kv_start + s.kv_cols].T
        ms = slice(s.mlp_start, s.mlp_start + s.mlp_cols)
        wdown = L["w_down"][ms].T  # [H, I_loc]
        if i_pad != s.mlp_cols:
            wdown = np.concatenate([wdown, np.zeros((wdown.shape[0], i_pad - s.mlp_cols), np.float32)], 1)
        layers.append(LayerDeviceWeights(
            wqkv=t(np.concatenate([q, k, v], 0)),
            wo=t(L["w_o"][s.q_start:s.q_start + s.q_cols].T),
            wgu=interleave_gate_up(t(L["w_gate"][:, ms].T), t(L["w_up"][:, ms].T), i_pad),
            wdown=t(wdown),
            attn_norm=t(L["attn_norm"]), mlp_norm=t(L["mlp_norm"]),
        ))
    return DeviceWeights(config=cfg, layout=s, vocab_start=v0, vocab_local=vn, i_pad=i_pad,
                         embedding=t(w.embedding[v0:v0 + vn]), final_norm=t(w.final_norm),
                         lm_head=t(w.lm_head[:, v0:v0 + vn].T), layers=layers)


def synthetic_device_weights(cfg: ModelConfig, rank: int, world: int, seed: int = 0, std: float = 0.02,
                             device="cuda", dtype=torch.bfloat16, norm_noise: bool = False) -> DeviceWeights:
    """Random N(0, std) weights generated directly on ``device`` in device layout.

    Every rank draws the same full tensor from a per-(seed, layer, name) generator and keeps its
    slice, so shards of different TP degrees are slices of one model.
    """
    cfg.validate()
    s = shard_layout(cfg, rank, world)
    i_pad = pad_to(s.mlp_cols, GU_BLOCK)
    v0, vn = even_split(cfg.vocab_size, world, rank)
    H, I, V = cfg.hidden_dim, cfg.intermediate_size, cfg.vocab_size
    dev = torch.device(device)

    def full(name, rows, cols, li=-1):
        g = torch.Generator(device=dev)
        g.manual_seed(_seed_for(seed, li, name))
        x = torch.empty(rows, cols, device=dev, dtype=torch.float32)
        x.normal_(0.0, std, generator=g)
        return x

    def norm(name, li=-1):
        if not norm_noise:
            return torch.ones(H, device=dev, dtype=dtype)
        return (1.0 + full(name, 1, H, li)[0]).to(dtype)

    layers = []
    for li in range(cfg.num_layers):
        # rows = output features ([out, in] layout)
        wq = full("w_q", H, H, li)[s.q_start:s.q_start + s.q_cols]
        wk = full("w_k", cfg.kv_dim, H, li)[s.kv_start:s.kv_start + s.kv_cols]
        wv = full("w_v", cfg.kv_dim, H, li)[s.kv_start:s.kv_start + s.kv_cols]
        wqkv = torch.cat([wq, wk, wv]).to(dtype).contiguous()
        del wq, wk, wv
        wo = full("w_o", H, H, li)[:, s.q_start:s.q_start + s.q_cols].to(dtype).contiguous()
        ms = slice(s.mlp_start, s.mlp_start + s.mlp_cols)
        wg = full("w_gate", I, H, li)[ms].to(dtype)
        wu = full("w_up", I, H, li)[ms].to(dtype)
        wgu = interleave_gate_up(wg, wu, i_pad)
        del wg, wu
        wd = full("w_down", H, I, li)[:, ms].to(dtype)
        if i_pad != s.mlp_cols:
            wd = torch.cat([wd, torch.zeros(H, i_pad - s.mlp_cols, device=dev, dtype=dtype)], 1)
        layers.append(LayerDeviceWeights(wqkv=wqkv, wo=wo, wgu=wgu, wdown=wd.contiguous(),
                                         attn_norm=norm("attn_norm", li), mlp_norm=norm("mlp_norm", li)))
    emb = full("embedding", V, H)[v0:v0 + vn].to(dtype).contiguous()  # vocabulary-parallel (all rows at TP=1)
    head = full("lm_head", V, H)[v0:v0 + vn].to(dtype).contiguous()
    return DeviceWeights(config=cfg, layout=s, vocab_start=v0, vocab_local=vn, i_pad=i_pad,
                         embedding=emb, final_norm=norm("final_norm"), lm_head=head, layers=layers)
