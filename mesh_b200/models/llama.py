"""Tensor-parallel Llama decoder for one rank, built from the sm_100a kernels.

Per layer (reference ``forward_layer``, ``agent/src/inference/forward_pass.rs:1946-2025``):

    qkv   = tcgen05 GEMM(normed, wqkv)                    (swap-AB for decode-sized T)
    q     = RoPE(q); k,v -> paged KV pool                 (decode: in the qkv GEMM epilogue;
                                                          prefill: rope_kv_write)
    attn  = paged GQA attention                           (decode: split-KV; prefill: flash)
    part  = tcgen05 GEMM(attn, wo)                        -> own slot of the symmetric workspace
    resid, normed = AR(part) + resid, RMSNorm(mlp_norm)   (ar_fused_norm over NVLink; TP=1: add_rmsnorm;
                                                          opt-in at decode: one launch, gemm_allreduce_norm)
    h     = tcgen05 GEMM(normed, wgu) with SiLU(gate)*up epilogue
    part  = tcgen05 GEMM(h, wdown)
    resid, normed = AR(part) + resid, RMSNorm(next attn_norm or final_norm)

then lm_head (vocab-parallel, fp32 logits) and greedy argmax merged across ranks. The reference
computes full-vocab logits on every rank and samples on the host (forward_pass.rs:2028-2039).
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass
from typing import List, Optional

import torch
import torch.distributed as dist

from .. import ops
from ..config import EngineConfig, ModelConfig
from .weights import DeviceWeights


# MESH_NVTX=1: host NVTX ranges per layer and for the LM head (for nsys/ncu timelines).
# MESH_POISON=1: fill activation scratch with NaN before each step (catches unwritten outputs).
_NVTX = os.environ.get("MESH_NVTX", "0") == "1"
_POISON = os.environ.get("MESH_POISON", "0") == "1"


def _nvtx_range(name):
    """Open an NVTX range (name) or close the innermost one (None); no-op unless MESH_NVTX=1."""
    if not _NVTX:
        return
    if name is None:
        torch.cuda.nvtx.range_pop()
    else:
        torch.cuda.nvtx.range_push(name)


# Smallest half of a prefill chunk that runs overlapped with the other half (the SM-pair GEMM's
# minimum, so neither half falls back to the one-SM kernel's shared stream-K workspace).
PREFILL_SPLIT_MIN_TOKENS = 512


class KVPool:
    """Paged KV pool of one rank: K and V tensors [layers, pages, kv_heads_local, page_size, D] bf16.
    Page 0 is reserved as a scratch page for padded batch slots."""

    def __init__(self, cfg: ModelConfig, local_kv_heads: int, num_pages: int, page_size: int, device):
        shape = (cfg.num_layers, num_pages, local_kv_heads, page_size, cfg.head_dim)
        self.k = torch.zeros(shape, dtype=torch.bfloat16, device=device)
        self.v = torch.zeros(shape, dtype=torch.bfloat16, device=device)
        self.num_pages = num_pages
        self.page_size = page_size

    @staticmethod
    def bytes_per_page(cfg: ModelConfig, local_kv_heads: int, page_size: int) -> int:
        return 2 * cfg.num_layers * local_kv_heads * page_size * cfg.head_dim * 2


@dataclass
class StepMeta:
    """Device metadata of one forward."""
    ids: torch.Tensor            # [T] int32
    pos: torch.Tensor            # [T] int32
    slot: torch.Tensor           # [T] int64 page*page_size + offset (-1: no KV write)
    block_tables: torch.Tensor   # [S, max_pages] int32
    seq_lens: torch.Tensor       # [S] int32 keys per sequence after this step
    cu_q: Optional[torch.Tensor] = None     # [S+1] int32 (prefill)
    last_idx: Optional[torch.Tensor] = None  # [S] int64 rows whose logits are needed (prefill)
    max_q_len: int = 1
    decode: bool = True
    # per-row sampling parameters (fp32 [S]: 1/T with 0 = greedy, top_p, threshold r); None = greedy
    inv_t: Optional[torch.Tensor] = None
    top_p: Optional[torch.Tensor] = None
    thr: Optional[torch.Tensor] = None
    nucleus: bool = True   # some row has 0 < top_p < 1 (the sampler's radix passes are needed)
    cu_host: Optional[List[int]] = None  # host copy of cu_q (prefill): lets the runner split the chunk


class LlamaRunner:
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
        c = self.cfg
        self.hq = weights.layout.local_q_heads
        self.hkv = weights.layout.local_kv_heads
        self.D = c.head_dim
        self.H = c.hidden_dim
        self.scale = 1.0 / math.sqrt(self.D)
        self.window = ecfg.sliding_window or 0
        self.cos, self.sin = ops.rope_tables(self.D, c.rope_base, max_pos or max(ecfg.max_seq_len, 8192) + 1,
                                             self.device)
        self.max_tokens = max_tokens
        self.symm = None
        self.use_fused_ar = self.world > 1 and ecfg.allreduce_impl != "nccl"
        # bound of every cross-rank wait inside the collective kernels (reference allreduce timeout)
        self.ar_timeout = float(ecfg.allreduce_timeout_s)
        # "push": the o_proj / down GEMM epilogues scatter partial rows to their owner ranks over
        # NVLink (fused GEMM -> reduce-scatter); otherwise GEMMs write locally and the AR kernel pulls
        self.push_rs = self.use_fused_ar and ecfg.allreduce_impl in ("push", "push_oneshot")
        # "gemm_ar": decode-sized steps run o_proj / down_proj with the all-reduce, residual add and
        # RMSNorm in the GEMM's own launch. Measured at TP2 it is slower than the GEMM followed by
        # the separate fused all-reduce kernel (decode step 3.93 vs 3.42 ms), so "auto" keeps the
        # separate kernel and the one-launch form is opt-in.
        self.gemm_ar = (self.use_fused_ar and ecfg.allreduce_impl == "gemm_ar" and self.H % 8 == 0 and
                        self.H <= 8192)
        if self.use_fused_ar:
            from ..parallel.symm import SymmWorkspace
            self.symm = SymmWorkspace(max_tokens, self.H, self.device, group, multicast=ecfg.nvls)
        # Prefill overlap: a chunk of several prompts runs as two halves on two streams, each with its
        # own symmetric workspace, so one half's all-reduces (NVLink, a few SMs) run while the other
        # half's GEMMs hold the tensor cores. Every all-reduce goes through one third stream, in the
        # same order on every rank: a GPU then never holds two all-reduce grids that wait on peers at
        # once (two such grids, each waiting for blocks the peer GPU could not schedule because its
        # SMs were held by the other one, stalled until their bounded waits ran out). Only with the
        # peer-memory all-reduce (NCCL calls on two streams could be ordered differently on
        # different ranks) and when both halves are big enough for the SM-pair GEMM, which uses no
        # shared workspace.
        self.overlap_prefill = (self.use_fused_ar and not self.push_rs and bool(ecfg.prefill_overlap)
                                and max_tokens >= 2 * PREFILL_SPLIT_MIN_TOKENS)
        self.symm2 = None
        self._streams = None
        self._comm = None
        self.split_steps = 0
        if self.overlap_prefill:
            from ..parallel.symm import SymmWorkspace
            self.symm2 = SymmWorkspace(max_tokens, self.H, self.device, group, multicast=ecfg.nvls)
            # two compute streams (one per half) and one stream that runs every all-reduce
            self._streams = (torch.cuda.Stream(self.device), torch.cuda.Stream(self.device))
            self._comm = torch.cuda.Stream(self.device)
        # vocabulary-parallel embedding: this rank's rows live in a table every peer maps, and each
        # token's row is read from its owner (one launch, fused with the first RMSNorm)
        self.emb_table = None
        if self.world > 1:
            if weights.embedding.shape[0] != weights.vocab_local:
                raise ValueError("TP>1 expects this rank's vocabulary rows of the embedding")
            from ..parallel.symm import SymmTable
            self.emb_table = SymmTable(weights.embedding, c.vocab_size, group)
            weights.embedding = self.emb_table.local
        self._cand_gather = None
        self._sampler = None
        # keep fp32 logits (tests, sampling); the greedy decode path fuses argmax into the LM head
        self.keep_logits = False
        self.last_logits = None

    # ------------------------------------------------------------------------------------------
    def _resid_normed(self, T: int, symm=None):
        symm = symm or self.symm
        if symm is not None:
            return symm.resid(T), symm.normed(T)
        return (torch.empty(T, self.H, dtype=torch.bfloat16, device=self.device),
                torch.empty(T, self.H, dtype=torch.bfloat16, device=self.device))

    def _two_shot(self, T: int) -> bool:
        impl = self.ecfg.allreduce_impl
        if impl in ("oneshot", "push_oneshot"):
            return False
        if impl == "twoshot":
            return True
        if self.push_rs:
            return T >= self.world  # pushing to the owner moves each row once; all-gather follows
        # one-shot reads every peer's full partial (T*H*2*(world-1) bytes per rank) behind one barrier;
        # two-shot moves 1/world of that each way behind two. Measured crossover on B200: two ranks
        # never (one-shot won up to T=4096 at H=4096), eight ranks between T=64 and T=512 at H=4096.
        if self.world <= 2:
            return False
        return T * self.H * 2 * (self.world - 1) > (8 << 20)

    def _reduce(self, part: torch.Tensor, resid: torch.Tensor, normed: torch.Tensor, gamma: torch.Tensor,
                parity: int, symm=None, comm=None):
        """resid += sum_ranks(part); normed = RMSNorm(resid) * gamma. With ``comm`` the all-reduce
        runs on that stream, ordered after the current stream's work and before its next."""
        if comm is not None:
            cur = torch.cuda.current_stream(self.device)
            comm.wait_stream(cur)
            with torch.cuda.stream(comm):
                self._reduce(part, resid, normed, gamma, parity, symm, comm)
            cur.wait_stream(comm)
            return
        T = resid.shape[0]
        eps = self.cfg.rms_norm_eps
        symm = symm or self.symm
        if self.world == 1:
            ops.add_rmsnorm(resid, gamma, normed, eps, delta=part)
        elif self.push_rs:
            symm.push_reduce_norm(T, parity, gamma, eps, two_shot=self._two_shot(T), timeout_s=self.ar_timeout)
        elif self.use_fused_ar:
            symm.fused_allreduce_norm(T, parity, gamma, eps, two_shot=self._two_shot(T), timeout_s=self.ar_timeout,
                                      multicast=self.world >= 8)
        else:  # NCCL baseline
            dist.all_reduce(part, group=self.group)
            ops.add_rmsnorm(resid, gamma, normed, eps, delta=part)

    def _push(self, T: int, parity: int):
        return self.symm.push_args(T, parity, self._two_shot(T)) if self.push_rs else None

    def _part_buf(self, T: int, parity: int, scratch: dict, symm=None) -> torch.Tensor:
        if self.use_fused_ar:
            return (symm or self.symm).partial(parity, T)
        key = ("part", T)
        if key not in scratch:
            scratch[key] = torch.empty(T, self.H, dtype=torch.bfloat16, device=self.device)
        return scratch[key]

    def _proj_reduce(self, x: torch.Tensor, wt: torch.Tensor, resid: torch.Tensor, normed: torch.Tensor,
                     gamma: torch.Tensor, parity: int, bufs: dict, symm=None, comm=None):
        """resid += sum_ranks(x @ wt.T); normed = RMSNorm(resid) * gamma (row-parallel projection)."""
        T = x.shape[0]
        if self.gemm_ar and T <= ops.SWAP_AB_MAX_TOKENS:
            self.symm.gemm_allreduce_norm(x, wt, parity, gamma, self.cfg.rms_norm_eps, timeout_s=self.ar_timeout,
                                          multicast=self.world >= 8)
            return
        part = self._part_buf(T, parity, bufs, symm)
        ops.linear(x, wt, out=part, push=self._push(T, parity))
        self._reduce(part, resid, normed, gamma, parity, symm, comm)

    # ------------------------------------------------------------------------------------------
    def _embed(self, m: StepMeta, resid: torch.Tensor, normed: torch.Tensor) -> None:
        c, w = self.cfg, self.w
        if self.emb_table is not None:
            ops.embed_peer_norm(self.emb_table.bases, m.ids, c.vocab_size, w.layers[0].attn_norm, c.rms_norm_eps,
                                resid, normed)
        else:
            ops.embedding(m.ids, w.embedding, resid)
            ops.add_rmsnorm(resid, w.layers[0].attn_norm, normed, c.rms_norm_eps)

    def _scratch(self, T: int, buf) -> tuple:
        w = self.w
        qkv = buf("qkv", (T, (self.hq + 2 * self.hkv) * self.D))
        q = buf("q", (T, self.hq * self.D))
        attn = buf("attn", (T, self.hq * self.D))
        h = buf("h", (T, w.i_pad))
        if _POISON:
            # debug: NaN in every activation scratch buffer, so a kernel that skips part of its
            # output shows up as NaN in the result instead of reusing the previous step's values
            for t in (qkv, q, attn, h):
                t.fill_(float("nan"))
        return qkv, q, attn, h

    def _layer(self, li: int, m: StepMeta, resid, normed, scr: tuple, bufs: dict, symm=None, comm=None) -> None:
        """One decoder layer; ``normed`` holds this layer's attention-normed input on entry and the
        next layer's (or the final norm's) on exit. Each layer runs two all-reduces, so the
        partial-buffer parity is the same (0 then 1) in every layer."""
        w = self.w
        L = w.layers[li]
        qkv, q, attn, h = scr
        kc, vc = self.kv.k[li], self.kv.v[li]
        ops.qkv_rope(normed, L.wqkv, m.pos, m.slot, self.cos, self.sin, q, kc, vc, self.hq, self.hkv, qkv_buf=qkv)
        if m.decode:
            ops.attn_decode(q, kc, vc, m.block_tables, m.seq_lens, attn, self.scale, self.window,
                            max_len_hint=m.max_q_len)
        else:
            ops.attn_prefill(q, kc, vc, m.cu_q, m.seq_lens, m.block_tables, attn, m.max_q_len, self.scale,
                             self.window)
        self._proj_reduce(attn, L.wo, resid, normed, L.mlp_norm, 0, bufs, symm, comm)
        ops.linear(normed, L.wgu, out=h, epi=ops.EPI_SILU_BF16)
        gamma = w.layers[li + 1].attn_norm if li + 1 < len(w.layers) else w.final_norm
        self._proj_reduce(h, L.wdown, resid, normed, gamma, 1, bufs, symm, comm)

    def _split_point(self, m: StepMeta) -> int:
        """Number of prompts in the first half of a prefill chunk run as two overlapped halves, or 0
        to run it whole: the prompt boundary closest to half the tokens that leaves both halves
        at least PREFILL_SPLIT_MIN_TOKENS tokens."""
        if not self.overlap_prefill or m.decode or m.cu_host is None or len(m.cu_host) < 3:
            return 0
        cu = m.cu_host
        T = cu[-1]
        best, best_d = 0, None
        for k in range(1, len(cu) - 1):
            a = cu[k]
            if a >= PREFILL_SPLIT_MIN_TOKENS and T - a >= PREFILL_SPLIT_MIN_TOKENS:
                d = abs(2 * a - T)
                if best_d is None or d < best_d:
                    best, best_d = k, d
        return best

    @staticmethod
    def _sub_meta(m: StepMeta, k0: int, k1: int) -> StepMeta:
        """Prompts [k0, k1) of a prefill chunk as a step of their own (row and index tensors rebased)."""
        cu = m.cu_host
        r0, r1 = cu[k0], cu[k1]
        cu_q = m.cu_q[k0:k1 + 1] if r0 == 0 else m.cu_q[k0:k1 + 1] - r0
        last = None if m.last_idx is None else (m.last_idx[k0:k1] if r0 == 0 else m.last_idx[k0:k1] - r0)
        return StepMeta(ids=m.ids[r0:r1], pos=m.pos[r0:r1], slot=m.slot[r0:r1], block_tables=m.block_tables[k0:k1],
                        seq_lens=m.seq_lens[k0:k1], cu_q=cu_q, last_idx=last,
                        max_q_len=max(cu[i + 1] - cu[i] for i in range(k0, k1)), decode=False,
                        cu_host=[c - r0 for c in cu[k0:k1 + 1]])

    def forward(self, m: StepMeta, bufs: Optional[dict] = None) -> torch.Tensor:
        """Run all layers and the LM head; returns next-token ids [S] (int32, greedy)."""
        w = self.w
        bufs = {} if bufs is None else bufs
        T = m.ids.shape[0]
        if T > self.max_tokens:
            raise ValueError(f"step of {T} tokens exceeds runner capacity {self.max_tokens}")

        def mkbuf(store):
            def buf(name, shape, dtype=torch.bfloat16):
                key = (name, tuple(shape), dtype)
                t = store.get(key)
                if t is None:
                    t = store[key] = torch.empty(shape, dtype=dtype, device=self.device)
                return t
            return buf

        buf = mkbuf(bufs)
        rng = _nvtx_range
        k = self._split_point(m)
        if k:
            # two halves on two streams, layer by layer, each with its own symmetric workspace
            self.split_steps += 1
            halves = [(self._sub_meta(m, 0, k), self.symm, {}),
                      (self._sub_meta(m, k, len(m.cu_host) - 1), self.symm2, {})]
            main = torch.cuda.current_stream(self.device)
            states = []
            for (hm, sy, hb), st in zip(halves, self._streams):
                st.wait_stream(main)
                with torch.cuda.stream(st):
                    r, n = self._resid_normed(hm.ids.shape[0], sy)
                    self._embed(hm, r, n)
                    states.append((hm, sy, hb, st, r, n, self._scratch(hm.ids.shape[0], mkbuf(hb))))
            for li in range(len(w.layers)):
                rng(f"layer {li}")
                for hm, sy, hb, st, r, n, scr in states:
                    with torch.cuda.stream(st):
                        self._layer(li, hm, r, n, scr, hb, sy, self._comm)
                rng(None)
            for state in states:
                main.wait_stream(state[3])
            rng("lm_head")
            S = m.last_idx.shape[0]
            final = buf("final", (S, self.H))
            sa = states[0][0].last_idx.shape[0]
            torch.index_select(states[0][5], 0, states[0][0].last_idx, out=final[:sa])
            torch.index_select(states[1][5], 0, states[1][0].last_idx, out=final[sa:])
            return self._lm_head(m, final, S, buf, rng)

        resid, normed = self._resid_normed(T)
        self._embed(m, resid, normed)
        scr = self._scratch(T, buf)
        for li in range(len(w.layers)):
            rng(f"layer {li}")
            self._layer(li, m, resid, normed, scr, bufs)
            rng(None)

        rng("lm_head")
        if m.last_idx is not None:
            S = m.last_idx.shape[0]
            final = buf("final", (S, self.H))
            torch.index_select(normed, 0, m.last_idx, out=final)
        else:
            final, S = normed, T
        return self._lm_head(m, final, S, buf, rng)

    def _lm_head(self, m: StepMeta, final: torch.Tensor, S: int, buf, rng) -> torch.Tensor:
        w = self.w
        cand = buf("cand", (S, 2), torch.float32)
        sampled = m.inv_t is not None
        if self.keep_logits or sampled or S > ops.SWAP_AB_MAX_TOKENS:
            logits = buf("logits", (S, w.vocab_local), torch.float32)
            ops.linear(final, w.lm_head, out=logits, epi=ops.EPI_STORE_F32)
            ops.argmax_partial(logits, w.vocab_start, cand)
            self.last_logits = logits
        else:
            tiles = buf("cand_tiles", ((w.vocab_local + 127) // 128, S, 2), torch.float32)
            ops.lm_head_argmax(final, w.lm_head, w.vocab_start, tiles, cand)
        ids_out = buf("next_ids", (S,), torch.int32)
        greedy = buf("greedy_ids", (S,), torch.int32) if sampled else ids_out
        if self.world == 1:
            ops.argmax_merge(cand.view(1, S, 2), greedy)
        else:
            gathered = buf("cand_all", (self.world, S, 2), torch.float32)
            dist.all_gather_into_tensor(gathered.view(-1), cand.view(-1), group=self.group)
            ops.argmax_merge(gathered, greedy)
        if sampled:
            # temperature / top-p rows on the device over this rank's vocabulary slice
            self.sampler(S).sample(logits, m.inv_t, m.top_p, m.thr, greedy, w.vocab_start, ids_out,
                                   nucleus=m.nucleus)
        rng(None)
        return ids_out

    def sampler(self, rows: int):
        """The device sampler of this runner (buffers for at least ``rows`` rows)."""
        from ..ops.sampling import DeviceSampler
        if self._sampler is None or self._sampler.B < rows:
            self._sampler = DeviceSampler(max(rows, 64), self.device, self.group, self.world, self.rank)
        return self._sampler
