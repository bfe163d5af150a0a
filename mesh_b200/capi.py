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
    """Call the C entry point on the current stream; returns its status code (0 = launched)."""
    B = q.shape[0]
    D = k_cache.shape[3]
    return lib().mesh_attn_decode_noalloc(
        q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), block_tables.data_ptr(), seq_lens.data_ptr(),
        out.data_ptr(), B, q.shape[1] // D, k_cache.shape[1], D, k_cache.shape[2], block_tables.shape[1], splits,
        float(scale), window, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
