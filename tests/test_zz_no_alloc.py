"""The allocation-free C entry point (``mesh_attn_decode_noalloc``) against the regular op and the
plain fp32 attention reference.

It serves callers that cannot allocate device memory at call time (their memory is already
owned by a pool, or they run where cudaMalloc/cudaFree are not allowed); its split-KV scratch
is a fixed array inside the library. The entry point is called through its exported C symbol
(ctypes) twice in a row. The first call is the larger one (more sequences, more splits), so the
second, smaller call runs over scratch that still holds the first call's values: a result that
read a stale slot would differ from the reference. Each result is compared with the PyTorch op
on the same inputs and with an fp32 softmax(QK^T)V over the gathered pages. This file is named to
be collected last.
"""
import ctypes
import math

import pytest
import torch

from mesh_b200 import capi, ops
from mesh_b200.ops import reference as ref

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


def _fp32_reference(q, kc, vc, bt, lens, scale, window):
    """softmax(q k^T * scale) v in fp32 over each sequence's pages, gathered in block-table order."""
    B, hkv, ps, D = q.shape[0], kc.shape[1], kc.shape[2], kc.shape[3]
    hq = q.shape[1] // D
    out = torch.empty(B, hq, D, dtype=torch.float32, device=q.device)
    for i, L in enumerate(lens):
        pages = bt[i, :(L + ps - 1) // ps].long()
        k = kc[pages].permute(0, 2, 1, 3).reshape(-1, hkv, D)[:L]
        v = vc[pages].permute(0, 2, 1, 3).reshape(-1, hkv, D)[:L]
        out[i] = ref.attention(q[i].view(1, hq, D), k, v, torch.tensor([L - 1], device=q.device),
                               torch.arange(L, device=q.device), scale, window)[0]
    return out.view(B, hq * D)


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm()).item()


def test_symbol_is_exported():
    L = capi.lib()
    assert isinstance(L.mesh_attn_decode_noalloc, ctypes._CFuncPtr)


@pytest.mark.parametrize("G,D,window", [(4, 128, 0), (8, 128, 0), (4, 64, 50)])
def test_noalloc_matches_op_and_fp32_two_calls(G, D, window):
    hkv = 2
    scale = 1.0 / math.sqrt(D)
    # call 1: 6 sequences x 4 splits; call 2: 3 sequences x 2 splits over the scratch call 1 left
    plan = [(11, [1, 40, 333, 1024, 97, 512], 4), (12, [700, 5, 129], 2)]
    for call, (seed, lens, splits) in enumerate(plan):
        q, kc, vc, bt, sl = _case(seed, len(lens), hkv, G, D, lens)
        want = torch.empty_like(q)
        ops.attn_decode(q, kc, vc, bt, sl, want, scale, window, splits=splits, impl="simt")
        got = torch.full_like(q, float("nan"))
        rc = capi.attn_decode_noalloc(q, kc, vc, bt, sl, got, splits, scale, window)
        assert rc == 0, f"call {call}: status {rc}"
        torch.cuda.synchronize()
        assert torch.isfinite(got.float()).all(), call
        assert _rel(got, want) < 1e-2, (call, "vs op")
        gold = _fp32_reference(q, kc, vc, bt, lens, scale, window)
        assert _rel(got, gold) < 2e-2, (call, "vs fp32")


def test_noalloc_rejects_oversized_request():
    q, kc, vc, bt, sl = _case(3, 64, 8, 4, 128, [64] * 64)
    out = torch.zeros_like(q)
    # 64 * 32 heads * 8 splits * 129 floats > 1 Mi floats
    rc = capi.attn_decode_noalloc(q, kc, vc, bt, sl, out, 8, 0.088, 0)
    assert rc == -2
    torch.cuda.synchronize()
    assert out.abs().sum() == 0  # nothing launched


def test_noalloc_wrapper_rejects_bad_inputs():
    q, kc, vc, bt, sl = _case(4, 2, 2, 4, 128, [10, 20])
    out = torch.zeros_like(q)
    with pytest.raises(ValueError):
        capi.attn_decode_noalloc(q.float(), kc, vc, bt, sl, out, 1, 0.088, 0)
    with pytest.raises(ValueError):
        capi.attn_decode_noalloc(q, kc, vc, bt.long(), sl, out, 1, 0.088, 0)
    with pytest.raises(ValueError):
        capi.attn_decode_noalloc(q, kc, vc, bt.t(), sl, out, 1, 0.088, 0)
