"""Per-kernel microbenchmark on the shapes of one decoder step.

    python -m mesh_b200.utils.opbench --model llama3-8b --tp 1 --batch 64 --ctx 576 --prefill 4096

Each kernel is timed with CUDA events after warm-up; operands rotate through enough copies to
exceed the 126 MB L2, so every timed launch reads its weights from HBM. Achieved bandwidth and
FLOP rate are reported against the measured peaks in MEASURED_PEAKS.json when present.
"""
from __future__ import annotations

import argparse
import json
import math
import os

import torch

from .. import ops
from ..config import get_preset
from ..models.sharding import shard_layout, even_split
from ..models.weights import GU_BLOCK, pad_to

L2_BYTES = 126 * 1024 * 1024


def peaks():
    p = os.path.join(os.path.dirname(__file__), "..", "..", "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return d["hbm_gbs"], d["bf16_tflops"], "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, 1590.0, "fallback"


def timeit(fn, iters=20, warmup=3):
    """Device time per call in microseconds. The timed calls are captured once in a CUDA graph and
    replayed, so host launch overhead does not count (as in the CUDA-graph decode step)."""
    for i in range(warmup):
        fn(i)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):
        with torch.cuda.graph(g):
            for i in range(iters):
                fn(i + 1)
    torch.cuda.current_stream().wait_stream(st)
    g.replay()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    g.replay()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters * 1e3


def copies_for(nbytes):
    return max(2, math.ceil(2 * L2_BYTES / max(nbytes, 1)))


def bench_linear(name, T, N, K, epi, rows, hbm, tf):
    dev = "cuda"
    w_bytes = N * K * 2
    nc = min(copies_for(w_bytes), 64)
    ws = [torch.randn(N, K, device=dev).mul_(0.02).to(torch.bfloat16) for _ in range(nc)]
    x = torch.randn(T, K, device=dev).to(torch.bfloat16)
    n_out = N // 2 if epi == ops.EPI_SILU_BF16 else N
    out = torch.empty(T, n_out, device=dev, dtype=torch.float32 if epi == ops.EPI_STORE_F32 else torch.bfloat16)
    us = timeit(lambda i: ops.linear(x, ws[i % nc], out=out, epi=epi))
    # the same product through cuBLAS (plain bf16 output, no fused epilogue), for reference
    ref_out = torch.empty(T, N, device=dev, dtype=torch.bfloat16)
    us_cublas = timeit(lambda i: torch.mm(x, ws[i % nc].t(), out=ref_out))
    byts = w_bytes + T * K * 2 + out.numel() * out.element_size()
    flops = 2.0 * T * N * K
    rows.append(dict(op=name, shape=f"T={T} N={N} K={K}", us=round(us, 2), GBps=round(byts / us / 1e3, 1),
                     TFLOPs=round(flops / us / 1e6, 1), hbm_frac=round(byts / us / 1e3 / hbm, 3),
                     tc_frac=round(flops / us / 1e6 / tf, 3), cublas_us=round(us_cublas, 2)))
    del ws


def trace_gemms(cfg, s, T, modes=(0, 1)):
    """Run each decode GEMM with %globaltimer stamps and summarise its phases (us after the
    earliest CTA start): griddep wait passed, first MMA data, last MMA issued, epilogue done, exit;
    for stream-K tiles also the contributor/owner fixup steps. mode 0 = auto schedule, 1 = whole
    tiles only."""
    dev = "cuda"
    H = cfg.hidden_dim
    i_pad = pad_to(s.mlp_cols, GU_BLOCK)
    for name, N, K, epi in [("qkv", s.q_cols + 2 * s.kv_cols, H, 0), ("o_proj", H, s.q_cols, 0),
                            ("gate_up", 2 * i_pad, H, 2), ("down", H, i_pad, 0)]:
        w = torch.randn(N, K, device=dev).mul_(0.02).to(torch.bfloat16)
        xin = torch.randn(T, K, device=dev).to(torch.bfloat16)
        out = torch.empty(T, N // 2 if epi == 2 else N, device=dev, dtype=torch.bfloat16)
        for mode in modes:
            tr = torch.zeros(148 * 32, dtype=torch.int64, device=dev)
            for _ in range(3):
                ops.gemm(w, xin, out, epi, trans=True, trace=tr, mode=mode)
            torch.cuda.synchronize()
            t = tr.view(-1, 32).cpu()
            t = t[t[:, 0] > 0]
            t0 = t[:, 0].min()
            rel = (t - t0).double() / 1e3
            med = lambda c: round(float(rel[:, c].median()), 2)
            mx = lambda c: round(float(rel[:, c].max()), 2)
            contrib = rel[t[:, 8] > 0]
            owner = rel[t[:, 12] > 0]
            cm = lambda x, c: round(float(x[:, c].median()), 2) if len(x) else None
            plan = ops.ext().gemm_plan(N, T, K, epi, True, torch.cuda.current_device())
            print(json.dumps(dict(trace=name, mode=mode, plan=list(plan), ctas=len(t), start_max=mx(0), waited=med(1),
                                  first_data_med=med(3), mma_done_med=med(4), mma_done_max=mx(4),
                                  epi_start_med=med(5), epi_fetched_med=med(12), epi_stored_med=med(13),
                                  epi_done_max=mx(6), exit_max=mx(7), contrib_n=len(contrib),
                                  contrib_partial_written=cm(contrib, 8), contrib_flag_set=cm(contrib, 9),
                                  owner_n=len(owner), owner_wait_done=cm(owner, 10),
                                  owner_bulk_landed=cm(owner, 12), owner_add0=cm(owner, 13),
                                  owner_fin0=cm(owner, 14), owner_done=cm(owner, 11),
                                  ck_first_sum=med(11) if plan[7] > 1 else None)))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="llama3-8b")
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--ctx", type=int, default=576)
    ap.add_argument("--prefill", type=int, default=4096)
    ap.add_argument("--json", default="")
    ap.add_argument("--trace", action="store_true", help="per-CTA phase timestamps of the decode GEMMs")
    a = ap.parse_args()
    cfg = get_preset(a.model)
    s = shard_layout(cfg, 0, a.tp)
    hbm, tf, src = peaks()
    rows = []
    H, D = cfg.hidden_dim, cfg.head_dim
    qkv_n = s.q_cols + 2 * s.kv_cols
    i_pad = pad_to(s.mlp_cols, GU_BLOCK)
    _, v_loc = even_split(cfg.vocab_size, a.tp, 0)
    for T in (a.batch, a.prefill):
        tag = "decode" if T == a.batch else "prefill"
        bench_linear(f"{tag}.qkv", T, qkv_n, H, ops.EPI_STORE_BF16, rows, hbm, tf)
        bench_linear(f"{tag}.o_proj", T, H, s.q_cols, ops.EPI_STORE_BF16, rows, hbm, tf)
        bench_linear(f"{tag}.gate_up+silu", T, 2 * i_pad, H, ops.EPI_SILU_BF16, rows, hbm, tf)
        bench_linear(f"{tag}.down", T, H, i_pad, ops.EPI_STORE_BF16, rows, hbm, tf)
    bench_linear("decode.lm_head", a.batch, v_loc, H, ops.EPI_STORE_F32, rows, hbm, tf)

    # decode attention: B sequences of ctx keys, pages shuffled
    dev = "cuda"
    B, ps = a.batch, 16
    hkv, hq = s.local_kv_heads, s.local_q_heads
    pages_per = (a.ctx + ps - 1) // ps
    npages = B * pages_per + 1
    kv_bytes = npages * hkv * ps * D * 2 * 2
    nc = min(copies_for(kv_bytes), 16)
    kcs = [torch.randn(npages, hkv, ps, D, device=dev).to(torch.bfloat16) for _ in range(nc)]
    vcs = [torch.randn(npages, hkv, ps, D, device=dev).to(torch.bfloat16) for _ in range(nc)]
    bt = (torch.randperm(npages - 1, device=dev)[:B * pages_per] + 1).view(B, pages_per).int()
    lens = torch.full((B,), a.ctx, dtype=torch.int32, device=dev)
    q = torch.randn(B, hq * D, device=dev).to(torch.bfloat16)
    out = torch.empty_like(q)
    byts = B * a.ctx * hkv * D * 2 * 2
    for impl in ("tc", "simt"):
        us = timeit(lambda i: ops.attn_decode(q, kcs[i % nc], vcs[i % nc], bt, lens, out, 1 / math.sqrt(D),
                                              impl=impl))
        rows.append(dict(op=f"decode.attention[{impl}]", shape=f"B={B} ctx={a.ctx} hq={hq} hkv={hkv}",
                         us=round(us, 2), GBps=round(byts / us / 1e3, 1), hbm_frac=round(byts / us / 1e3 / hbm, 3)))
    del kcs, vcs
    # prefill attention: sequences of 512 tokens
    P = 512
    nseq = max(1, a.prefill // P)
    pp = P // ps
    np2 = nseq * pp + 1
    kc = torch.randn(np2, hkv, ps, D, device=dev).to(torch.bfloat16)
    vc = torch.randn(np2, hkv, ps, D, device=dev).to(torch.bfloat16)
    bt2 = (torch.arange(nseq * pp, device=dev) + 1).view(nseq, pp).int()
    qp = torch.randn(nseq * P, hq * D, device=dev).to(torch.bfloat16)
    op = torch.empty_like(qp)
    cu = torch.arange(0, nseq + 1, device=dev, dtype=torch.int32) * P
    kl = torch.full((nseq,), P, dtype=torch.int32, device=dev)
    us = timeit(lambda i: ops.attn_prefill(qp, kc, vc, cu, kl, bt2, op, P, 1 / math.sqrt(D)))
    flops = 4.0 * nseq * hq * D * P * P / 2
    rows.append(dict(op="prefill.attention", shape=f"{nseq}x{P} causal hq={hq}", us=round(us, 2),
                     TFLOPs=round(flops / us / 1e6, 1), tc_frac=round(flops / us / 1e6 / tf, 3)))
    # norm / rope
    for T in (a.batch, a.prefill):
        r = torch.randn(T, H, device=dev).to(torch.bfloat16)
        d = torch.randn(T, H, device=dev).to(torch.bfloat16)
        g = torch.ones(H, device=dev, dtype=torch.bfloat16)
        n = torch.empty_like(r)
        us = timeit(lambda i: ops.add_rmsnorm(r, g, n, 1e-5, delta=d))
        rows.append(dict(op="add_rmsnorm", shape=f"T={T} H={H}", us=round(us, 2),
                         GBps=round(T * H * 2 * 4 / us / 1e3, 1)))
    # fused greedy LM head (argmax in the GEMM epilogue) vs logits + separate argmax
    nc = min(copies_for(v_loc * H * 2), 64)
    heads = [torch.randn(v_loc, H, device=dev).mul_(0.02).to(torch.bfloat16) for _ in range(nc)]
    xh = torch.randn(a.batch, H, device=dev).to(torch.bfloat16)
    tiles = torch.empty((v_loc + 127) // 128, a.batch, 2, device=dev)
    cand = torch.empty(a.batch, 2, device=dev)
    us = timeit(lambda i: ops.lm_head_argmax(xh, heads[i % nc], 0, tiles, cand))
    rows.append(dict(op="decode.lm_head+argmax(fused)", shape=f"T={a.batch} V={v_loc} H={H}", us=round(us, 2),
                     GBps=round(v_loc * H * 2 / us / 1e3, 1), hbm_frac=round(v_loc * H * 2 / us / 1e3 / hbm, 3)))
    del heads
    for row in rows:
        print(json.dumps(row))
    print(json.dumps({"peaks": {"hbm_gbs": hbm, "bf16_tflops": tf, "source": src}}))
    if a.trace:
        trace_gemms(cfg, s, a.batch)
    if a.json:
        with open(a.json, "w") as f:
            json.dump(rows, f, indent=1)


if __name__ == "__main__":
    main()
