"""Baseline B: a plain PyTorch bf16 tensor-parallel forward of the same decoder.

This is the comparison arm for the sm_100a kernels, built only from library code:

* linears are ``torch.nn.functional.linear`` (cuBLAS/cuBLASLt);
* RMSNorm is ``torch.nn.functional.rms_norm``; RoPE, SiLU and the residual adds are torch ops;
* the paged KV pool is written with index assignment and read back by gathering each sequence's
  pages into a contiguous [B, kv_heads, S, D] tensor; decode attention is two batched matmuls with
  a masked fp32 softmax between them, prefill uses ``scaled_dot_product_attention`` (causal).
  This is the shape of the reference's own attention path, which concatenates its pages and
  applies an explicit mask every step (``forward_pass.rs:633-680``, ``:2811-2835``);
* the two per-layer tensor-parallel reductions are ``torch.distributed.all_reduce`` (NCCL), as in
  the reference's forward layer (``forward_pass.rs:1974-2010``) but over NVLink instead of TCP;
* the LM head is vocab-parallel; the greedy token is each rank's ``max`` merged through an NCCL
  all-gather.

``TorchTPRunner`` has the interface of ``models.llama.LlamaRunner`` (``forward(StepMeta, bufs)``
returning next-token ids), so the same ``Engine`` drives it: same scheduling, same chunked
prefill, same CUDA-graph decode buckets. Only the compute path differs. It reads the same
``DeviceWeights`` (the gate/up rows interleaved in blocks of 64 are split with a view).
"""
from __future__ import annotations

import math
from typing import Optional

import torch
import torch.distributed as dist
import torch.nn.functional as F

from .. import ops
from ..config import EngineConfig
from ..models.llama import KVPool, StepMeta
from ..models.weights import GU_BLOCK, DeviceWeights


def _rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Half-split rotation of x [T, heads, D] with cos/sin [T, D/2] (fp32 math, bf16 result)."""
    half = x.shape[-1] // 2
    xf = x.float()
    l, r = xf[..., :half], xf[..., half:]
    c, s = cos[:, None, :], sin[:, None, :]
    return torch.cat([l * c - r * s, l * s + r * c], -1).to(x.dtype)


class TorchTPRunner:
    def __init__(self, weights: DeviceWeights, ecfg: EngineConfig, kv: KVPool, device, group=None,
                 max_tokens: int = 8192, max_pos: int = 0):
        self.w = weights
        self.cfg = weights.config
        self.ecfg = ecfg
        self.kv = kv
        self.device = torch.device(device)
        self.group = group
        self.world = weights.layout.world
        self.rank = weights.layout.rank
        self.hq = weights.layout.local_q_heads
        self.hkv = weights.layout.local_kv_heads
        self.D = self.cfg.head_dim
        self.H = self.cfg.hidden_dim
        self.scale = 1.0 / math.sqrt(self.D)
        self.window = ecfg.sliding_window or 0
        self.cos, self.sin = ops.rope_tables(self.D, self.cfg.rope_base,
                                             max_pos or max(ecfg.max_seq_len, 8192) + 1, self.device)
        self.max_tokens = max_tokens
        self.keep_logits = False
        self.last_logits = None

    # ------------------------------------------------------------------------------------------
    def _all_reduce(self, x: torch.Tensor):
        if self.world > 1:
            dist.all_reduce(x, group=self.group)

    def _write_kv(self, kc, vc, k, v, slot):
        """k/v [T, hkv, D] into pages; slot -1 (padded decode rows) goes to the scratch page 0."""
        ps = self.kv.page_size
        s = torch.where(slot < 0, torch.zeros_like(slot), slot)
        page, off = s // ps, s % ps
        kc[page, :, off] = k
        vc[page, :, off] = v

    def _attn_decode(self, q, kc, vc, m: StepMeta):
        """Gather each sequence's pages, then grouped-query attention as two batched matmuls (the q
        heads of one KV head form the rows of one [G, S] score block, so K/V are not repeated per
        q head) with an fp32 masked softmax between them."""
        B = q.shape[0]
        bt = m.block_tables.long()
        ps = self.kv.page_size
        S = bt.shape[1] * ps
        G = self.hq // self.hkv
        K = kc[bt].permute(0, 2, 1, 3, 4).reshape(B, self.hkv, S, self.D)
        V = vc[bt].permute(0, 2, 1, 3, 4).reshape(B, self.hkv, S, self.D)
        kpos = torch.arange(S, device=q.device)
        lens = m.seq_lens.long()[:, None]
        mask = kpos[None, :] < lens
        if self.window > 0:
            mask &= kpos[None, :] >= lens - self.window
        sc = torch.matmul(q.view(B, self.hkv, G, self.D), K.transpose(-1, -2)).float() * self.scale
        sc = sc.masked_fill(~mask[:, None, None, :], float("-inf"))
        pr = torch.softmax(sc, -1).to(q.dtype)
        return torch.matmul(pr, V).reshape(B, self.hq * self.D)

    def _attn_prefill(self, q, kc, vc, m: StepMeta):
        T = q.shape[0]
        ps = self.kv.page_size
        out = torch.empty(T, self.hq * self.D, dtype=q.dtype, device=q.device)
        cu = m.cu_q.tolist()
        klens = m.seq_lens.tolist()
        for i, kl in enumerate(klens):
            a, b = cu[i], cu[i + 1]
            ql = b - a
            pages = m.block_tables[i, :(kl + ps - 1) // ps].long()
            K = kc[pages].permute(1, 0, 2, 3).reshape(self.hkv, -1, self.D)[:, :kl]
            V = vc[pages].permute(1, 0, 2, 3).reshape(self.hkv, -1, self.D)[:, :kl]
            qi = q[a:b].view(ql, self.hq, self.D).transpose(0, 1)
            if ql == kl and self.window == 0:
                o = F.scaled_dot_product_attention(qi[None], K[None], V[None], is_causal=True, scale=self.scale,
                                                   enable_gqa=True)[0]
            else:
                qpos = torch.arange(kl - ql, kl, device=q.device)[:, None]
                kpos = torch.arange(kl, device=q.device)[None, :]
                mask = kpos <= qpos
                if self.window > 0:
                    mask &= kpos > qpos - self.window
                o = F.scaled_dot_product_attention(qi[None], K[None], V[None], attn_mask=mask[None, None],
                                                   scale=self.scale, enable_gqa=True)[0]
            out[a:b] = o.transpose(0, 1).reshape(ql, self.hq * self.D)
        return out

    # ------------------------------------------------------------------------------------------
    def forward(self, m: StepMeta, bufs: Optional[dict] = None) -> torch.Tensor:
        c, w = self.cfg, self.w
        T = m.ids.shape[0]
        if T > self.max_tokens:
            raise ValueError(f"step of {T} tokens exceeds runner capacity {self.max_tokens}")
        H, eps, D = self.H, c.rms_norm_eps, self.D
        if self.world == 1:
            resid = F.embedding(m.ids.long(), w.embedding)
        else:
            # vocabulary-parallel embedding: rows this rank holds, zeros elsewhere, summed over ranks
            local = m.ids.long() - w.vocab_start
            hit = (local >= 0) & (local < w.vocab_local)
            resid = F.embedding(local.clamp(0, w.vocab_local - 1), w.embedding) * hit[:, None].to(w.embedding.dtype)
            dist.all_reduce(resid, group=self.group)
        normed = F.rms_norm(resid, (H,), w.layers[0].attn_norm, eps)
        pos = m.pos.long()
        cos, sin = self.cos[pos], self.sin[pos]
        nq, nkv = self.hq * D, self.hkv * D
        for li, L in enumerate(w.layers):
            kc, vc = self.kv.k[li], self.kv.v[li]
            qkv = F.linear(normed, L.wqkv)
            q = _rope(qkv[:, :nq].view(T, self.hq, D), cos, sin)
            k = _rope(qkv[:, nq:nq + nkv].view(T, self.hkv, D), cos, sin)
            v = qkv[:, nq + nkv:].view(T, self.hkv, D)
            self._write_kv(kc, vc, k, v, m.slot)
            q = q.reshape(T, nq)
            attn = self._attn_decode(q, kc, vc, m) if m.decode else self._attn_prefill(q, kc, vc, m)
            part = F.linear(attn, L.wo)
            self._all_reduce(part)
            resid = resid + part
            normed = F.rms_norm(resid, (H,), L.mlp_norm, eps)
            gu = F.linear(normed, L.wgu).view(T, -1, 2, GU_BLOCK)
            h = (F.silu(gu[:, :, 0]) * gu[:, :, 1]).reshape(T, -1)
            part = F.linear(h, L.wdown)
            self._all_reduce(part)
            resid = resid + part
            gamma = w.layers[li + 1].attn_norm if li + 1 < len(w.layers) else w.final_norm
            normed = F.rms_norm(resid, (H,), gamma, eps)
        final = normed.index_select(0, m.last_idx) if m.last_idx is not None else normed
        logits = F.linear(final, w.lm_head).float()
        if self.keep_logits:
            self.last_logits = logits
        val, idx = logits.max(-1)
        idx = idx + w.vocab_start
        if self.world == 1:
            return idx.to(torch.int32)
        S = final.shape[0]
        vals = torch.empty(self.world, S, dtype=val.dtype, device=val.device)
        idxs = torch.empty(self.world, S, dtype=idx.dtype, device=idx.device)
        dist.all_gather_into_tensor(vals.view(-1), val.contiguous(), group=self.group)
        dist.all_gather_into_tensor(idxs.view(-1), idx.contiguous(), group=self.group)
        best = vals.argmax(0)  # first maximum: the lowest rank, i.e. the lowest vocabulary index
        return idxs.gather(0, best[None])[0].to(torch.int32)
