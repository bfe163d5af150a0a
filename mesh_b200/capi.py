"""ctypes access to the allocation-free C entry point ``mesh_attn_decode_noalloc``
(``libmesh_noalloc.so``, built in-tree next to this file).

The entry point runs split-KV paged decode attention with its scratch in a fixed device array of
the library (4 MiB per device), for callers that cannot allocate device memory while they run:
runtimes that own all GPU memory through their own pool, real-time loops where cudaMalloc and
cudaFree are not allowed, and plain C hosts. The first call on a device resolves the scratch
array's address and must come before any CUDA stream capture on that device; calls that overlap
on the GPU race on the shared scratch. This interface has no counterpart in the reference.
"""
from __future__ import annotations

import ctypes
import os

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libmesh_noalloc.so")
SCRATCH_FLOATS = 1 << 20
_LIB = None


def lib():
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is not built; run __graft_entry__.build()")
        L = ctypes.CDLL(LIB_PATH)
        f = L.mesh_attn_decode_noalloc
        f.restype = ctypes.c_int
        f.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_int] * 7 + [ctypes.c_float, ctypes.c_int, ctypes.c_void_p]
        _LIB = L
    return _LIB


def attn_decode_noalloc(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, block_tables: torch.Tensor,
                        seq_lens: torch.Tensor, out: torch.Tensor, splits: int, scale: float, window: int = 0) -> int:
    """Call the C entry point on the current stream of the tensors' device; returns its status
    code (0 = launched). The C side takes the device from the current CUDA device, so the call is
    made with ``q``'s device current and on that device's current stream."""
    bf16 = [("q", q), ("k_cache", k_cache), ("v_cache", v_cache), ("out", out)]
    i32 = [("block_tables", block_tables), ("seq_lens", seq_lens)]
    for name, t in bf16 + i32:
        if not t.is_cuda:
            raise ValueError(f"attn_decode_noalloc: {name} must be a CUDA tensor")
        if t.device != q.device:
            raise ValueError(f"attn_decode_noalloc: {name} is on {t.device}, q on {q.device}")
        if not t.is_contiguous():
            raise ValueError(f"attn_decode_noalloc: {name} must be contiguous")
    for name, t in bf16:
        if t.dtype != torch.bfloat16:
            raise ValueError(f"attn_decode_noalloc: {name} must be bf16, got {t.dtype}")
    for name, t in i32:
        if t.dtype != torch.int32:
            raise ValueError(f"attn_decode_noalloc: {name} must be int32, got {t.dtype}")
    if q.dim() != 2 or out.shape != q.shape or k_cache.dim() != 4 or v_cache.shape != k_cache.shape:
        raise ValueError("attn_decode_noalloc: q/out [B, Hq*D], k/v cache [pages, Hkv, page, D]")
    B = q.shape[0]
    D = k_cache.shape[3]
    with torch.cuda.device(q.device):
        stream = torch.cuda.current_stream(q.device).cuda_stream
        return lib().mesh_attn_decode_noalloc(
            q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), block_tables.data_ptr(), seq_lens.data_ptr(),
            out.data_ptr(), B, q.shape[1] // D, k_cache.shape[1], D, k_cache.shape[2], block_tables.shape[1],
            splits, float(scale), window, ctypes.c_void_p(stream))
