"""Numerics of every sm_100a kernel against a plain fp32 PyTorch reference of the same op."""
import math

import pytest
import torch

from mesh_b200 import ops
from mesh_b200.ops import reference as ref

pytestmark = pytest.mark.gpu
DEV = "cuda"


def rel_err(x, y):
    x, y = x.float(), y.float()
    return ((x - y).norm() / (y.norm() + 1e-6)).item()


@pytest.fixture(autouse=True)
def _check_err():
    yield
    ops.scratch(torch.device("cuda", torch.cuda.current_device())).check("kernel")


def _rand(*shape, std=1.0, dtype=torch.bfloat16, seed=0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return (torch.randn(*shape, generator=g, device=DEV) * std).to(dtype)


# ------------------------------------------------------------------------------------------ GEMM
@pytest.mark.parametrize("M,N,K", [(128, 128, 64), (256, 512, 1024), (300, 200, 328), (1, 384, 4096),
                                   (64, 6144, 4096), (17, 1000, 512), (4096, 1024, 2048)])
@pytest.mark.parametrize("trans", [False, True])
def test_gemm_bf16(M, N, K, trans):
    x = _rand(M, K, seed=1)
    w = _rand(N, K, std=0.05, seed=2)
    want = x.float() @ w.float().T
    if trans:  # weights on the MMA M side: out^T = w @ x^T
        out = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
        ops.gemm(w, x, out, ops.EPI_STORE_BF16, trans=True)
    else:
        out = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
        ops.gemm(x, w, out, ops.EPI_STORE_BF16, trans=False)
    torch.cuda.synchronize()
    assert rel_err(out, want) < 1e-2


@pytest.mark.parametrize("mode", [0, 1, 2])
@pytest.mark.parametrize("trans", [False, True])
def test_gemm_f32_schedules(mode, trans):
    M, N, K = 64, 768, 2048
    x = _rand(M, K, seed=3)
    w = _rand(N, K, std=0.05, seed=4)
    want = x.float() @ w.float().T
    out = torch.empty(M, N, dtype=torch.float32, device=DEV)
    if trans:
        ops.gemm(w, x, out, ops.EPI_STORE_F32, trans=True, mode=mode)
    else:
        ops.gemm(x, w, out, ops.EPI_STORE_F32, trans=False, mode=mode)
    torch.cuda.synchronize()
    assert rel_err(out, want) < 2e-3
    # counters must be left at zero so graph replays and later calls work
    assert int(ops.scratch(torch.device(DEV, 0)).gemm_counters.abs().sum()) == 0


@pytest.mark.parametrize("T", [1, 8, 64, 200, 1024])
def test_gemm_silu_mul(T):
    K, I = 1024, 512
    x = _rand(T, K, seed=5)
    w = _rand(2 * I, K, std=0.05, seed=6)
    y = x.float() @ w.float().T
    want = ref.silu_mul_interleaved(y)
    out = ops.linear(x, w, epi=ops.EPI_SILU_BF16)
    torch.cuda.synchronize()
    assert out.shape == (T, I)
    assert rel_err(out, want) < 1e-2


@pytest.mark.parametrize("M,N,K", [(4096, 6144, 4096), (1000, 1536, 512), (64, 28672, 1024)])
@pytest.mark.parametrize("epi", [0, 2])
def test_gemm_stream_k_matches_data_parallel(M, N, K, epi):
    """Stream-K tail waves and whole-tile scheduling give identical results (fixed reduction order)."""
    x = _rand(M, K, seed=14)
    w = _rand(N, K, std=0.05, seed=15)
    n_out = N // 2 if epi == 2 else N
    o1 = torch.empty(M, n_out, dtype=torch.bfloat16, device=DEV)
    o2 = torch.empty_like(o1)
    trans = M <= 256
    A, B = (w, x) if trans else (x, w)
    ops.gemm(A, B, o1, epi, trans=trans, mode=1)
    ops.gemm(A, B, o2, epi, trans=trans, mode=2)
    torch.cuda.synchronize()
    want = x.float() @ w.float().T
    if epi == 2:
        want = ref.silu_mul_interleaved(want)
    assert rel_err(o1, want) < 1e-2 and rel_err(o2, want) < 1e-2
    o3 = torch.empty_like(o1)
    ops.gemm(A, B, o3, epi, trans=trans, mode=2)
    torch.cuda.synchronize()
    assert torch.equal(o2, o3)  # deterministic


@pytest.mark.parametrize("M,N,K", [(768, 64, 4096), (6144, 64, 4096), (4096, 17, 512), (3584, 64, 4096),
                                   (300, 8, 1024), (128, 1, 256), (1024, 128, 2048)])
@pytest.mark.parametrize("epi", [0, 1, 2])
def test_gemm_cluster_split_k(M, N, K, epi):
    """Cluster split-K (swap-AB: M weight rows, N tokens): every CTA of a cluster accumulates a
    share of the k-range and the shares are summed through distributed shared memory."""
    if epi == 2 and M % 128:
        pytest.skip("SiLU epilogue needs the feature dim % 128")
    w = _rand(M, K, std=0.05, seed=21)
    x = _rand(N, K, seed=22)
    want = x.float() @ w.float().T
    if epi == 2:
        want = ref.silu_mul_interleaved(want)
    dt = torch.float32 if epi == 1 else torch.bfloat16
    out = torch.empty(N, want.shape[1], dtype=dt, device=DEV)
    ops.gemm(w, x, out, epi, trans=True, mode=3)
    torch.cuda.synchronize()
    assert rel_err(out, want) < (2e-3 if epi == 1 else 1e-2)
    again = torch.empty_like(out)
    ops.gemm(w, x, again, epi, trans=True, mode=3)
    torch.cuda.synchronize()
    assert torch.equal(out, again)  # fixed summation order


@pytest.mark.parametrize("V,T", [(4096, 64), (16032, 64), (1000, 5)])
def test_lm_head_argmax_cluster_split(V, T):
    """Fused greedy head on shapes that take the cluster split-K schedule."""
    H = 4096
    w = _rand(V, H, std=0.05, seed=23)
    x = _rand(T, H, seed=24)
    logits = x.float() @ w.float().T
    tiles = torch.empty((V + 127) // 128, T, 2, dtype=torch.float32, device=DEV)
    out = torch.empty(T, 2, dtype=torch.float32, device=DEV)
    ops.lm_head_argmax(x, w, 0, tiles, out)
    torch.cuda.synchronize()
    idx = out[:, 1].contiguous().view(torch.int32).long()
    picked = logits.gather(1, idx[:, None])[:, 0]
    # the chosen entry is the max up to bf16 rounding of the accumulated logits
    assert bool((picked >= logits.max(-1).values - 2e-2 * logits.abs().max()).all())


@pytest.mark.parametrize("trans", [False, True])
@pytest.mark.parametrize("epi", [0, 1, 2])
def test_gemm_whole_tile_epilogue_strided_out(trans, epi):
    """Whole-tile (data-parallel) epilogue into a column slice of a wider tensor: an output pitch
    that is not a multiple of 16 bytes takes the scalar store path."""
    T, N, K = 200, 512, 256
    x = _rand(T, K, seed=25)
    w = _rand(N, K, std=0.05, seed=26)
    want = x.float() @ w.float().T
    if epi == 2:
        want = ref.silu_mul_interleaved(want)
    n_out = want.shape[1]
    dt = torch.float32 if epi == 1 else torch.bfloat16
    big = torch.zeros(T, n_out + 3, dtype=dt, device=DEV)
    out = big[:, 1:1 + n_out]
    A, B = (w, x) if trans else (x, w)
    ops.gemm(A, B, out, epi, trans=trans, mode=1)
    torch.cuda.synchronize()
    assert rel_err(out, want) < (2e-3 if epi == 1 else 1e-2)
    assert float(big[:, 0].abs().max()) == 0.0 and float(big[:, -2:].abs().max()) == 0.0


def test_linear_both_orientations_agree():
    x = _rand(100, 512, seed=7)
    w = _rand(640, 512, std=0.05, seed=8)
    a = ops.linear(x, w, swap_ab=True)
    b = ops.linear(x, w, swap_ab=False)
    torch.cuda.synchronize()
    assert rel_err(a, b) < 1e-2


# ------------------------------------------------------------------------------------- norm etc.
@pytest.mark.parametrize("H", [256, 4096, 8192])
def test_add_rmsnorm(H):
    T = 33
    resid = _rand(T, H, seed=9)
    delta = _rand(T, H, seed=10)
    gamma = (1 + 0.1 * _rand(H, seed=11).float()).to(torch.bfloat16)
    want_resid = (resid.float() + delta.float()).to(torch.bfloat16)
    want = ref.rmsnorm(want_resid.float(), gamma, 1e-5)
    normed = torch.empty_like(resid)
    r = resid.clone()
    ops.add_rmsnorm(r, gamma, normed, 1e-5, delta=delta)
    torch.cuda.synchronize()
    assert torch.equal(r, want_resid)
    assert rel_err(normed, want) < 1e-2
    r2 = resid.clone()
    ops.add_rmsnorm(r2, gamma, normed, 1e-5)
    assert rel_err(normed, ref.rmsnorm(resid.float(), gamma, 1e-5)) < 1e-2


def test_rope_kv_write():
    T, hq, hkv, D, ps, pages = 40, 8, 2, 128, 16, 10
    qkv = _rand(T, (hq + 2 * hkv) * D, seed=12)
    pos = torch.arange(100, 100 + T, dtype=torch.int32, device=DEV)
    page_ids = torch.tensor([3, 7, 1], device=DEV)
    p = torch.arange(T, device=DEV)
    slot = (page_ids[p // ps] * ps + p % ps).to(torch.int64)
    slot[5] = -1
    cos, sin = ops.rope_tables(D, 5e5, 4096, DEV)
    kc = torch.zeros(pages, hkv, ps, D, dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros_like(kc)
    q = torch.empty(T, hq * D, dtype=torch.bfloat16, device=DEV)
    ops.rope_kv_write(qkv, pos, slot, cos, sin, q, kc, vc, hq, hkv)
    torch.cuda.synchronize()
    qr = ref.rope(qkv[:, :hq * D], pos, D, 5e5)
    kr = ref.rope(qkv[:, hq * D:(hq + hkv) * D], pos, D, 5e5)
    assert rel_err(q, qr) < 1e-2
    for t in range(T):
        if t == 5:
            continue
        pg, off = int(page_ids[t // ps]), t % ps
        assert rel_err(kc[pg, :, off].reshape(-1), kr[t]) < 1e-2
        assert torch.equal(vc[pg, :, off].reshape(-1), qkv[t, (hq + hkv) * D:])
    assert kc[page_ids[0], :, 5].abs().sum() == 0  # slot -1 skipped


@pytest.mark.parametrize("T,hq,hkv", [(40, 8, 2), (64, 32, 8), (64, 4, 1), (7, 8, 8)])
@pytest.mark.parametrize("mode", [0, 1, 2, 3])
def test_qkv_rope_fused_matches_gemm_then_rope(T, hq, hkv, mode):
    """Decode qkv GEMM with RoPE and the paged KV write in its epilogue == GEMM + rope_kv_write, for
    every schedule (auto, whole tiles, stream-K, cluster split-K), including a padding slot (-1)."""
    H, D, ps, pages = 1024, 128, 16, 12
    if mode == 3 and ((hq + 2 * hkv) >= 148):
        pytest.skip("cluster split-K needs fewer tiles than SMs")
    x = _rand(T, H, seed=31)
    w = _rand((hq + 2 * hkv) * D, H, std=0.05, seed=32)
    pos = torch.arange(200, 200 + T, dtype=torch.int32, device=DEV)
    page_ids = torch.tensor([3, 7, 1, 9, 11], device=DEV)
    p = torch.arange(T, device=DEV)
    slot = (page_ids[p // ps] * ps + p % ps).to(torch.int64)
    slot[T // 2] = -1
    cos, sin = ops.rope_tables(D, 5e5, 4096, DEV)
    kc1 = torch.zeros(pages, hkv, ps, D, dtype=torch.bfloat16, device=DEV)
    vc1, kc2, vc2 = torch.zeros_like(kc1), torch.zeros_like(kc1), torch.zeros_like(kc1)
    q1 = torch.empty(T, hq * D, dtype=torch.bfloat16, device=DEV)
    q2 = torch.empty_like(q1)
    ops.qkv_rope(x, w, pos, slot, cos, sin, q1, kc1, vc1, hq, hkv, mode=mode if mode else 0)
    qkv = torch.empty(T, w.shape[0], dtype=torch.bfloat16, device=DEV)
    ops.linear(x, w, out=qkv)
    ops.rope_kv_write(qkv, pos, slot, cos, sin, q2, kc2, vc2, hq, hkv)
    torch.cuda.synchronize()
    # against an fp32 reference of the whole op, and against the unfused kernels
    y = x.float() @ w.float().T
    qr = ref.rope(y[:, :hq * D], pos, D, 5e5)
    assert rel_err(q1, qr) < 1e-2
    assert rel_err(q1, q2) < 1e-2
    assert rel_err(kc1, kc2) < 1e-2 and rel_err(vc1, vc2) < 1e-2
    t = T // 2
    pg, off = int(page_ids[t // ps]), t % ps
    assert kc1[pg, :, off].abs().sum() == 0 and vc1[pg, :, off].abs().sum() == 0  # slot -1 skipped


def test_embedding_and_argmax():
    V, H = 1000, 256
    table = _rand(V, H, seed=13)
    ids = torch.tensor([0, 5, 999, 17], dtype=torch.int32, device=DEV)
    out = torch.empty(4, H, dtype=torch.bfloat16, device=DEV)
    ops.embedding(ids, table, out)
    torch.cuda.synchronize()
    assert torch.equal(out, table[ids.long()])
    logits = torch.randn(5, 3000, device=DEV)
    logits[2, 100] = 50.0
    logits[2, 200] = 50.0  # tie: first index wins
    cand = torch.empty(5, 2, device=DEV)
    ops.argmax_partial(logits, 0, cand)
    idx = torch.empty(5, dtype=torch.int32, device=DEV)
    ops.argmax_merge(cand.view(1, 5, 2), idx)
    torch.cuda.synchronize()
    assert idx.tolist() == logits.argmax(-1).tolist()
    assert int(idx[2]) == 100
    # two "ranks" each holding half of the vocabulary
    c2 = torch.empty(2, 5, 2, device=DEV)
    ops.argmax_partial(logits[:, :1500].contiguous(), 0, c2[0])
    ops.argmax_partial(logits[:, 1500:].contiguous(), 1500, c2[1])
    ops.argmax_merge(c2, idx)
    torch.cuda.synchronize()
    assert idx.tolist() == logits.argmax(-1).tolist()


# -------------------------------------------------------------------------------------- attention
def _paged_kv(lens, hkv, D, ps, seed):
    """Random K/V for sequences of the given lengths scattered over shuffled pages."""
    npages = sum((L + ps - 1) // ps for L in lens) + 4
    g = torch.Generator().manual_seed(seed)
    perm = torch.randperm(npages - 1, generator=g) + 1
    kc = _rand(npages, hkv, ps, D, seed=seed + 1)
    vc = _rand(npages, hkv, ps, D, seed=seed + 2)
    maxp = max((L + ps - 1) // ps for L in lens)
    bt = torch.zeros(len(lens), maxp, dtype=torch.int32)
    k_list, v_list, c = [], [], 0
    for i, L in enumerate(lens):
        n = (L + ps - 1) // ps
        pg = perm[c:c + n]
        c += n
        bt[i, :n] = pg
        k_list.append(kc[pg.to(DEV)].permute(0, 2, 1, 3).reshape(-1, hkv, D)[:L])
        v_list.append(vc[pg.to(DEV)].permute(0, 2, 1, 3).reshape(-1, hkv, D)[:L])
    return kc, vc, bt.to(DEV), k_list, v_list


@pytest.mark.parametrize("G,D,impl", [(4, 128, "tc"), (8, 128, "tc"), (1, 128, "tc"), (2, 128, "tc"),
                                      (4, 128, "simt"), (8, 128, "simt"), (4, 64, "simt")])
@pytest.mark.parametrize("splits", [1, 3])
@pytest.mark.parametrize("window", [0, 100])
def test_attn_decode(G, D, impl, splits, window):
    lens = [1, 17, 300, 1029, 64]
    hkv, ps = 2, 16
    hq = hkv * G
    kc, vc, bt, ks, vs = _paged_kv(lens, hkv, D, ps, seed=20)
    q = _rand(len(lens), hq * D, seed=30)
    out = torch.empty_like(q)
    scale = 1 / math.sqrt(D)
    ops.attn_decode(q, kc, vc, bt, torch.tensor(lens, dtype=torch.int32, device=DEV), out, scale, window, splits=splits,
                    impl=impl)
    torch.cuda.synchronize()
    for i, L in enumerate(lens):
        want = ref.attention(q[i].view(1, hq, D), ks[i], vs[i], torch.tensor([L - 1], device=DEV),
                             torch.arange(L, device=DEV), scale, window)
        assert rel_err(out[i].view(1, hq, D), want) < 2e-2, (i, L)


@pytest.mark.parametrize("splits", [2, 5])
def test_attn_decode_in_kernel_combine(splits, monkeypatch):
    """Split decode attention merging its partials in the last CTA of each (sequence, KV head):
    bitwise equal to the separate combine kernel, the same on a repeated launch, and every arrival
    counter back at zero afterwards."""
    lens = [1, 17, 300, 1029, 64, 700]
    hkv, ps, G, D = 2, 16, 4, 128
    kc, vc, bt, ks, vs = _paged_kv(lens, hkv, D, ps, seed=21)
    q = _rand(len(lens), hkv * G * D, seed=31)
    sl = torch.tensor(lens, dtype=torch.int32, device=DEV)
    outs = []
    for fused in (True, True, False):
        monkeypatch.setattr(ops, "_FUSED_COMBINE", fused)
        out = torch.full_like(q, float("nan"))
        ops.attn_decode(q, kc, vc, bt, sl, out, 1 / math.sqrt(D), 0, splits=splits, impl="tc")
        torch.cuda.synchronize()
        outs.append(out)
    ops.scratch(DEV).check("attn_decode")
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])
    assert int(ops.scratch(DEV).attn_cnt.abs().sum()) == 0


@pytest.mark.parametrize("G", [4, 8, 1, 2])
@pytest.mark.parametrize("window", [0, 50])
@pytest.mark.parametrize("impl", ["tc", "fa2"])
def test_attn_prefill_varlen_prefix(G, window, impl):
    _prefill_case(G, window, impl, k_lens=[40, 300, 129, 64], q_lens=[40, 100, 1, 64], seed=40)


@pytest.mark.parametrize("G", [4, 8])
@pytest.mark.parametrize("q_mult", [1.0, 12.0])
def test_attn_prefill_tc_long_blocks(G, q_mult):
    """Several 128-key blocks per query tile, ragged ends, a cached prefix, and (q_mult 12) scores
    spread wide enough that the running maximum moves by more than 2^8 and O is rescaled in TMEM."""
    _prefill_case(G, 0, "tc", k_lens=[1500, 777, 256], q_lens=[700, 777, 129], seed=50, q_mult=q_mult)


def _prefill_case(G, window, impl, k_lens, q_lens, seed, q_mult=1.0):
    hkv, D, ps = 2, 128, 16
    hq = hkv * G
    kc, vc, bt, ks, vs = _paged_kv(k_lens, hkv, D, ps, seed=seed)
    T = sum(q_lens)
    q = (_rand(T, hq * D, seed=seed + 1).float() * q_mult).to(torch.bfloat16)
    out = torch.full_like(q, float("nan"))
    cu = torch.tensor([0] + list(torch.tensor(q_lens).cumsum(0)), dtype=torch.int32, device=DEV)
    scale = 1 / math.sqrt(D)
    ops.attn_prefill(q, kc, vc, cu, torch.tensor(k_lens, dtype=torch.int32, device=DEV), bt, out, max(q_lens), scale,
                     window, impl=impl)
    torch.cuda.synchronize()
    ops.scratch(DEV).check("attn_prefill")
    for i, (kl, ql) in enumerate(zip(k_lens, q_lens)):
        a = int(cu[i])
        qpos = torch.arange(kl - ql, kl, device=DEV)
        want = ref.attention(q[a:a + ql].view(ql, hq, D), ks[i], vs[i], qpos, torch.arange(kl, device=DEV), scale,
                             window)
        assert torch.isfinite(out[a:a + ql].float()).all(), (i, "rows not written")
        assert rel_err(out[a:a + ql].view(ql, hq, D), want) < 2e-2, i


@pytest.mark.parametrize("impl", ["tc", "fa2"])
def test_attn_prefill_batch_invariant(impl):
    """A sequence's prefill attention output does not depend on the other sequences of the batch:
    each sequence alone gives bitwise the same rows as the batch."""
    hkv, D, ps, G = 2, 128, 16, 4
    hq = hkv * G
    k_lens, q_lens = [5, 300, 17, 140], [5, 40, 17, 140]
    kc, vc, bt, ks, vs = _paged_kv(k_lens, hkv, D, ps, seed=60)
    T = sum(q_lens)
    q = _rand(T, hq * D, seed=61)
    cu = [0] + torch.tensor(q_lens).cumsum(0).tolist()
    scale = 1 / math.sqrt(D)
    out = torch.full_like(q, float("nan"))
    ops.attn_prefill(q, kc, vc, torch.tensor(cu, dtype=torch.int32, device=DEV),
                     torch.tensor(k_lens, dtype=torch.int32, device=DEV), bt, out, max(q_lens), scale, 0, impl=impl)
    for i, (kl, ql) in enumerate(zip(k_lens, q_lens)):
        qi = q[cu[i]:cu[i] + ql].clone()
        oi = torch.full_like(qi, float("nan"))
        ops.attn_prefill(qi, kc, vc, torch.tensor([0, ql], dtype=torch.int32, device=DEV),
                         torch.tensor([kl], dtype=torch.int32, device=DEV), bt[i:i + 1].contiguous(), oi, ql, scale,
                         0, impl=impl)
        torch.cuda.synchronize()
        assert torch.equal(oi, out[cu[i]:cu[i] + ql]), (impl, i)
