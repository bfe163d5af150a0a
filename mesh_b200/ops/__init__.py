"""Python front-end of the sm_100a kernels in ``mesh_b200._C``.

Every op here runs the hand-written CUDA kernel; there is no silent PyTorch fallback. If the
extension is missing on a machine with a GPU, ``ext()`` raises. ``mesh_b200.ops.reference``
holds plain fp32 PyTorch versions used only by tests as the numerical oracle.
"""
from __future__ import annotations

import os

import threading
from typing import Optional

import torch

_EXT = None
_LOCK = threading.Lock()

# Number of kernels launched through this module (a CUDA-graph replay re-launches the kernels
# counted while it was captured; callers multiply by replays).
LAUNCHES = [0]


def _count(n: int = 1):
    LAUNCHES[0] += n

EPI_STORE_BF16 = 0
EPI_STORE_F32 = 1
EPI_SILU_BF16 = 2
EPI_ARGMAX = 3
# decode-sized token counts use the swap-AB orientation (weights on the 128-row MMA side)
SWAP_AB_MAX_TOKENS = 256


def ext():
    """Import the compiled kernel module (built in-tree by ``__graft_entry__.build()``)."""
    global _EXT
    if _EXT is None:
        with _LOCK:
            if _EXT is None:
                try:
                    from .. import _C  # noqa: F401
                except ImportError as e:  # pragma: no cover - depends on the build
                    raise RuntimeError(
                        "mesh_b200._C is not built; run `python setup.py build_ext --inplace` "
                        "(or __graft_entry__.build()) before using the sm_100a kernels") from e
                _EXT = _C
    return _EXT


def available() -> bool:
    try:
        ext()
        return torch.cuda.is_available()
    except RuntimeError:
        return False


class DeviceScratch:
    """Per-device scratch shared by the ops of one stream: error word, GEMM split-K workspace and
    tile counters, split-KV attention scratch. Sized lazily; grows only outside graph capture."""

    def __init__(self, device):
        self.device = torch.device(device)
        self.err = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.gemm_ws = torch.empty(0, dtype=torch.float32, device=self.device)
        self.gemm_counters = torch.zeros(4096, dtype=torch.int32, device=self.device)
        self.attn_ws = torch.empty(0, dtype=torch.float32, device=self.device)
        # split decode attention: per-(sequence, KV head) arrival counters, zero between launches
        self.attn_cnt = torch.zeros(0, dtype=torch.int32, device=self.device)
        props = torch.cuda.get_device_properties(self.device)
        self.num_sms = props.multi_processor_count

    def ensure_gemm(self, floats: int, tiles: int):
        if self.gemm_ws.numel() < floats:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("GEMM workspace must be sized before CUDA graph capture")
            self.gemm_ws = torch.empty(max(floats, 1 << 20), dtype=torch.float32, device=self.device)
        if self.gemm_counters.numel() < tiles:
            self.gemm_counters = torch.zeros(tiles * 2, dtype=torch.int32, device=self.device)

    def ensure_attn(self, floats: int, counters: int = 0):
        if self.attn_ws.numel() < floats:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("attention scratch must be sized before CUDA graph capture")
            self.attn_ws = torch.empty(max(floats, 1 << 20), dtype=torch.float32, device=self.device)
        if self.attn_cnt.numel() < counters:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("attention scratch must be sized before CUDA graph capture")
            self.attn_cnt = torch.zeros(max(counters, 4096), dtype=torch.int32, device=self.device)

    def check(self, what: str = "kernel"):
        v = int(self.err.item())
        if v:
            self.err.zero_()
            self.attn_cnt.zero_()  # a launch that unwound early may have left counts behind
            raise RuntimeError(f"{what}: device error code {v} (1-3 pipeline wait timeout, 4 peer timeout, 5 bad argument)")


_SCRATCH = {}


def scratch(device=None) -> DeviceScratch:
    dev = torch.device(device if device is not None else torch.cuda.current_device())
    if dev.type == "cuda" and dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    s = _SCRATCH.get(dev)
    if s is None:
        s = _SCRATCH[dev] = DeviceScratch(dev)
    return s


def gemm(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor, epi: int = EPI_STORE_BF16, trans: bool = False,
         bn: int = 0, mode: int = 0, trace: Optional[torch.Tensor] = None, push: Optional[list] = None) -> torch.Tensor:
    """out = a @ b.T (trans=False, out [M, N']) or out^T = a @ b.T (trans=True, out [N, M'])
    with the tcgen05 kernel. a [M, K], b [N, K] bf16 K-contiguous. mode: 0 auto schedule,
    1 whole tiles only, 2 stream-K for the tail waves, 3 cluster split-K (swap-AB only)."""
    s = scratch(a.device)
    M, N, K = a.shape[0], b.shape[0], a.shape[1]
    if mode == 0 and bn == 0:
        key = (M, N, K, epi, trans, a.device.index)
        plan = _PLANS.get(key)
        if plan is None:
            plan = _PLANS[key] = ext().gemm_plan(M, N, K, epi, trans, a.device.index)
        if plan[2] > 0:
            s.ensure_gemm(plan[1], plan[2])
    else:
        # explicit schedule (tests): size the workspace for the worst case of this shape
        bn_ = bn or ext().gemm_plan(M, N, K, epi, trans, a.device.index)[0]
        tiles = ((M + 127) // 128) * ((N + bn_ - 1) // bn_)
        s.ensure_gemm((tiles + s.num_sms) * 128 * bn_, tiles)
    ext().gemm_tcgen05(a, b, out, epi, trans, bn, mode, s.gemm_ws, s.gemm_counters, s.err, trace, push or [])
    _count()
    return out


_PLANS = {}


def gemm_allreduce_norm(w: torch.Tensor, x: torch.Tensor, part_view: torch.Tensor, push: list, cfg: list,
                        gamma: torch.Tensor, eps: float, epoch: torch.Tensor, mode: int = 0,
                        trace: Optional[torch.Tensor] = None):
    """Swap-AB decode GEMM x @ w.T whose epilogue pushes partial rows to their owner ranks, with the
    tensor-parallel reduction, residual add, RMSNorm and all-gather of the normed rows in the same
    launch (``parallel.symm.SymmWorkspace.gemm_allreduce_norm`` builds the tables)."""
    s = scratch(x.device)
    M, N, K = w.shape[0], x.shape[0], w.shape[1]
    key = (M, N, K, EPI_STORE_BF16, True, x.device.index)
    plan = _PLANS.get(key)
    if plan is None:
        plan = _PLANS[key] = ext().gemm_plan(M, N, K, EPI_STORE_BF16, True, x.device.index)
    if mode != 0:
        # explicit schedule (tests): size the stream-K workspace for the worst case of this shape
        tiles = ((M + 127) // 128) * ((N + plan[0] - 1) // plan[0])
        s.ensure_gemm((tiles + s.num_sms) * 128 * plan[0], tiles)
    elif plan[2] > 0:
        s.ensure_gemm(plan[1], plan[2])
    ext().gemm_allreduce_norm(w, x, part_view, push, cfg, gamma, eps, epoch, mode, s.gemm_ws, s.gemm_counters, s.err,
                              trace)
    _count()


def linear(x: torch.Tensor, w: torch.Tensor, out: Optional[torch.Tensor] = None, epi: int = EPI_STORE_BF16,
           swap_ab: Optional[bool] = None, push: Optional[list] = None) -> torch.Tensor:
    """y = x @ w.T for x [T, K], w [N, K] (nn.Linear layout). Decode-sized T uses swap-AB so the
    weight rows fill the 128-row MMA tile; large T uses the normal orientation."""
    T, N = x.shape[0], w.shape[0]
    n_out = N // 2 if epi == EPI_SILU_BF16 else N
    if out is None:
        out = torch.empty(T, n_out, device=x.device, dtype=torch.float32 if epi == EPI_STORE_F32 else torch.bfloat16)
    if swap_ab is None:
        swap_ab = T <= SWAP_AB_MAX_TOKENS
    if swap_ab:
        return gemm(w, x, out, epi, trans=True, push=push)
    if (not push and _PAIR_GEMM and T >= PAIR_GEMM_MIN_TOKENS and epi in (EPI_STORE_BF16, EPI_SILU_BF16)
            and ext().gemm_2sm_supported(T, N, x.shape[1], epi)):
        return gemm_pair(x, w, out, epi)
    return gemm(x, w, out, epi, trans=False, push=push)


# Prefill-sized products run on SM pairs (256x512 tiles, tcgen05.mma.cta_group::2) from this many
# tokens: 1.34-1.51 PFLOP/s on the Llama-3-8B prefill shapes at T=4096 against 1.04-1.25 for the
# one-SM kernel. MESH_PAIR_GEMM=0 keeps the one-SM kernel everywhere (A/B measurements).
PAIR_GEMM_MIN_TOKENS = 512
_PAIR_GEMM = os.environ.get("MESH_PAIR_GEMM", "1") != "0"


def gemm_pair(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor, epi: int = EPI_STORE_BF16,
              trace: Optional[torch.Tensor] = None, tn: int = 0) -> torch.Tensor:
    """out = x @ w.T (EPI_SILU_BF16: SiLU(gate) * up of the interleaved gate/up product) on SM pairs.
    trace: optional int64 [384] of %globaltimer stamps for the first pair (producer empty-waits of both
    CTAs, then the MMA thread's full-waits). tn: tile width (128, 256 or 512 output columns per SM
    pair; 0: ``MESH_PAIR_TN`` if set, else 512 from N >= 1024 and 256 below)."""
    if tn:
        ext().gemm_2sm(x, w, out, epi, scratch(x.device).err, trace, tn)
    else:
        ext().gemm_2sm(x, w, out, epi, scratch(x.device).err, trace)
    _count()
    return out


def add_rmsnorm(resid: torch.Tensor, gamma: torch.Tensor, normed: torch.Tensor, eps: float,
                delta: Optional[torch.Tensor] = None):
    ext().add_rmsnorm(delta, resid, gamma, normed, eps)
    _count()
    return normed


EPI_QKV_ROPE = 4
# the fused decode qkv + RoPE + paged-KV-write GEMM; MESH_FUSED_QKV_ROPE=0 selects GEMM + rope_kv_write
_FUSED_QKV_ROPE = os.environ.get("MESH_FUSED_QKV_ROPE", "1") != "0"


def qkv_rope(x: torch.Tensor, wqkv: torch.Tensor, pos: torch.Tensor, slot: torch.Tensor, cos_t: torch.Tensor,
             sin_t: torch.Tensor, q_out: torch.Tensor, kcache: torch.Tensor, vcache: torch.Tensor, hq: int,
             hkv: int, qkv_buf: Optional[torch.Tensor] = None, mode: int = 0) -> torch.Tensor:
    """q = RoPE(x @ wq.T); k = RoPE(x @ wk.T) and v = x @ wv.T written into the paged KV pool at
    each token's slot. Decode-sized T with head_dim 128: one swap-AB GEMM whose epilogue applies
    RoPE and writes q and the pages directly. Otherwise: GEMM into `qkv_buf`, then rope_kv_write."""
    T = x.shape[0]
    if T <= SWAP_AB_MAX_TOKENS and kcache.shape[-1] == 128 and (_FUSED_QKV_ROPE or mode != 0):
        s = scratch(x.device)
        M, K = wqkv.shape
        if mode == 0:
            key = (M, T, K, EPI_QKV_ROPE, True, x.device.index)
            plan = _PLANS.get(key)
            if plan is None:
                plan = _PLANS[key] = ext().gemm_plan(M, T, K, EPI_QKV_ROPE, True, x.device.index)
            if plan[2] > 0:
                s.ensure_gemm(plan[1], plan[2])
        else:
            bn_ = ext().gemm_plan(M, T, K, EPI_QKV_ROPE, True, x.device.index)[0]
            tiles = ((M + 127) // 128) * ((T + bn_ - 1) // bn_)
            s.ensure_gemm((tiles + s.num_sms) * 128 * bn_, tiles)
        ext().gemm_qkv_rope(wqkv, x, q_out, pos, slot, cos_t, sin_t, kcache, vcache, hq, hkv, mode, s.gemm_ws,
                            s.gemm_counters, s.err)
        _count()
        return q_out
    if qkv_buf is None:
        qkv_buf = torch.empty(T, wqkv.shape[0], dtype=torch.bfloat16, device=x.device)
    linear(x, wqkv, out=qkv_buf)
    return rope_kv_write(qkv_buf, pos, slot, cos_t, sin_t, q_out, kcache, vcache, hq, hkv)


def rope_kv_write(qkv, pos, slot, cos_t, sin_t, q_out, kcache, vcache, hq: int, hkv: int):
    ext().rope_kv_write(qkv, pos, slot, cos_t, sin_t, q_out, kcache, vcache, hq, hkv)
    _count()
    return q_out


def embedding(ids: torch.Tensor, table: torch.Tensor, out: torch.Tensor):
    ext().embedding(ids, table, out, scratch(ids.device).err)
    _count()
    return out


# MESH_ATTN_FUSED_COMBINE=1: split decode attention merges its partials in the last CTA of each
# (sequence, KV head) instead of a separate combine launch. Measured at the TP8 decode shape (64 x 576
# keys, 1 KV head) it took 13.0 us against 8.9 us for the split kernel plus the combine launch (every
# CTA's device-wide fence and the serial merge cost more than the launch they save), so it is off.
_FUSED_COMBINE = os.environ.get("MESH_ATTN_FUSED_COMBINE", "0") == "1"


def attn_decode(q, kcache, vcache, block_tables, seq_lens, out, scale: float, window: int = 0,
                splits: int = 0, max_len_hint: int = 0, impl: str = "auto"):
    """Paged GQA decode attention. impl: "tc" (TMA-streamed, tensor-core fragments; head_dim 128,
    16-token pages), "simt" (CUDA-core variant, any page size, head_dim 64/128) or "auto"."""
    s = scratch(q.device)
    B, hkv, ps, D = q.shape[0], kcache.shape[1], kcache.shape[2], kcache.shape[3]
    hq = q.shape[1] // D
    if impl == "auto":
        impl = "tc" if (D == 128 and ps == 16) else "simt"
    if splits <= 0:
        splits = ext().attn_decode_pick_splits(B, hkv, max_len_hint or block_tables.shape[1] * ps, s.num_sms)
    fused = impl == "tc" and _FUSED_COMBINE
    if splits > 1:
        s.ensure_attn(B * hq * splits * (D + 1), B * hkv if fused else 0)
    if impl == "tc":
        ext().attn_decode_tc(q, kcache, vcache, block_tables, seq_lens, out, s.attn_ws, s.err, splits, scale, window,
                             s.attn_cnt if (fused and splits > 1) else None)
    else:
        ext().attn_decode(q, kcache, vcache, block_tables, seq_lens, out, s.attn_ws, splits, scale, window)
    _count(2 if (splits > 1 and not fused) else 1)
    return out


# MESH_PREFILL_ATTN=fa2 selects the mma.sync kernel (A/B measurements); the default is the tcgen05
# kernel wherever it serves the shape (head_dim 128, 16-token pages)
_PREFILL_IMPL = os.environ.get("MESH_PREFILL_ATTN", "tc")


def attn_prefill(q, kcache, vcache, cu_q, k_lens, block_tables, out, max_q_len: int, scale: float,
                 window: int = 0, impl: Optional[str] = None):
    """Causal paged varlen GQA attention of the new tokens of each sequence. impl: "tc" (tcgen05
    with TMEM accumulators; head_dim 128 and 16-token pages) or "fa2" (mma.sync, any page size)."""
    impl = impl or _PREFILL_IMPL
    D = kcache.shape[3]
    G = (q.shape[1] // D) // kcache.shape[1]
    if impl == "tc" and ext().attn_prefill_tc_supported(D, kcache.shape[2], G):
        ext().attn_prefill_tc(q, kcache, vcache, cu_q, k_lens, block_tables, out, max_q_len, scale, window,
                              scratch(q.device).err)
    else:
        ext().attn_prefill(q, kcache, vcache, cu_q, k_lens, block_tables, out, max_q_len, scale, window)
    _count()
    return out


def embed_peer_norm(bases: torch.Tensor, ids: torch.Tensor, vocab: int, gamma: torch.Tensor, eps: float,
                    resid: torch.Tensor, normed: torch.Tensor):
    """resid = embedding rows of ``ids`` read from the rank that owns each row (``bases``: the
    symmetric table of every rank), normed = RMSNorm(resid) * gamma. One launch."""
    ext().embed_peer_norm(bases, ids, vocab, gamma, eps, resid, normed, scratch(ids.device).err)
    _count()


def kv_pages_gather(k_pool: torch.Tensor, v_pool: torch.Tensor, pages, out: Optional[torch.Tensor] = None):
    """[layers, pages, hkv, ps, D] pools -> buffer [2, layers, len(pages), hkv*ps*D] (K then V)."""
    L, P = k_pool.shape[0], k_pool.shape[1]
    _check_pages(pages, P)
    page_elems = k_pool[0, 0].numel()
    if out is None:
        out = torch.empty(2, L, len(pages), page_elems, dtype=k_pool.dtype, device=k_pool.device)
    idx = torch.tensor(list(pages), dtype=torch.int32).pin_memory().to(k_pool.device, non_blocking=True)
    ext().kv_pages_copy(k_pool, v_pool, out, idx, True)
    _count()
    return out


def kv_pages_scatter(k_pool: torch.Tensor, v_pool: torch.Tensor, pages, buf: torch.Tensor):
    """Inverse of ``kv_pages_gather``: buffer rows go into ``pages`` of the pools (same device)."""
    _check_pages(pages, k_pool.shape[1])
    idx = torch.tensor(list(pages), dtype=torch.int32).pin_memory().to(k_pool.device, non_blocking=True)
    ext().kv_pages_copy(k_pool, v_pool, buf, idx, False)
    _count()


def _check_pages(pages, pool_pages: int):
    for p in pages:
        if not 0 <= int(p) < pool_pages:
            raise ValueError(f"page id {p} outside the pool of {pool_pages} pages")


def argmax_partial(logits: torch.Tensor, vocab_offset: int, out: torch.Tensor):
    ext().argmax_partial(logits, vocab_offset, out)
    _count()
    return out


def lm_head_argmax(x: torch.Tensor, w: torch.Tensor, vocab_offset: int, tiles_buf: torch.Tensor,
                   out: torch.Tensor) -> torch.Tensor:
    """Greedy head without materialising logits: the swap-AB GEMM epilogue keeps each token's max
    over every 128-row vocabulary tile, then one kernel reduces the tiles. out: [T, 2] float
    (value, global index bits)."""
    gemm(w, x, tiles_buf, EPI_ARGMAX, trans=True)
    ext().argmax_tiles(tiles_buf, vocab_offset, out)
    _count()
    return out


def argmax_merge(cand: torch.Tensor, ids: torch.Tensor):
    ext().argmax_merge(cand, ids)
    _count()
    return ids


def rope_tables(head_dim: int, base: float, max_pos: int, device) -> tuple:
    """cos/sin [max_pos, head_dim/2] fp32; inv_freq[i] = base^(-2i/d) computed in float64."""
    half = head_dim // 2
    inv = 1.0 / (torch.tensor(base, dtype=torch.float64) ** (torch.arange(half, dtype=torch.float64) * 2.0 / head_dim))
    t = torch.arange(max_pos, dtype=torch.float64)[:, None] * inv[None, :]
    return torch.cos(t).float().to(device), torch.sin(t).float().to(device)
