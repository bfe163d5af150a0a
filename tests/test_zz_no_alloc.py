"""The allocation-free C entry point (``mesh_attn_decode_noalloc``) against the regular op.

It serves callers that cannot allocate device memory at call time (their memory is already
owned by a pool, or they run where cudaMalloc/cudaFree are not allowed); its split-KV scratch
is a fixed array inside the library. The entry point is called through its exported C symbol
(ctypes) twice in a row and each result is compared with the PyTorch op's on the same inputs.
This file is named to be collected last.
"""
import ctypes
import math

import pytest
import torch

from mesh_b200 import capi, ops

pytestmark = pytest.mark.gpu


def _case(seed, B, hkv, G, D, lens, ps=16):
    g = torch.Generator(device="cuda").manual_seed(seed)
    maxp = max((L + ps - 1) // ps for L in lens)
    npages = B * maxp + 1
    kc = torch.randn(npages, hkv, ps, D, generator=g, device="cuda").to(torch.bfloat16)
    vc = torch.randn(npages, hkv, ps, D, generator=g, device="cuda").to(torch.bfloat16)
    perm = torch.randperm(npages - 1, generator=g, device="cuda")[:B * maxp] + 1
    bt = perm.view(B, maxp).int().contiguous()
    q = torch.randn(B, hkv * G * D, generator=g, device="cuda").to(torch.bfloat16)
    sl = torch.tensor(lens, dtype=torch.int32, device="cuda")
    return q, kc, vc, bt, sl


def test_symbol_is_exported():
    L = capi.lib()
    assert isinstance(L.mesh_attn_decode_noalloc, ctypes._CFuncPtr)


@pytest.mark.parametrize("G,D,splits,window", [(4, 128, 4, 0), (8, 128, 3, 0), (4, 64, 2, 50)])
def test_noalloc_matches_op_two_calls(G, D, splits, window):
    hkv = 2
    for call, seed in enumerate((11, 12)):  # two calls in a row share (and reuse) the scratch
        lens = [1, 40, 333, 1024, 97, 512][: 6]
        q, kc, vc, bt, sl = _case(seed, len(lens), hkv, G, D, lens)
        scale = 1.0 / math.sqrt(D)
        want = torch.empty_like(q)
        ops.attn_decode(q, kc, vc, bt, sl, want, scale, window, splits=splits, impl="simt")
        got = torch.full_like(q, float("nan"))
        rc = capi.attn_decode_noalloc(q, kc, vc, bt, sl, got, splits, scale, window)
        assert rc == 0, f"call {call}: status {rc}"
        torch.cuda.synchronize()
        assert torch.isfinite(got.float()).all()
        err = ((got.float() - want.float()).norm() / want.float().norm()).item()
        assert err < 1e-2, (call, err)


def test_noalloc_rejects_oversized_request():
    q, kc, vc, bt, sl = _case(3, 64, 8, 4, 128, [64] * 64)
    out = torch.zeros_like(q)
    # 64 * 32 heads * 8 splits * 129 floats > 1 Mi floats
    rc = capi.attn_decode_noalloc(q, kc, vc, bt, sl, out, 8, 0.088, 0)
    assert rc == -2
    torch.cuda.synchronize()
    assert out.abs().sum() == 0  # nothing launched
