"""Benchmarks of the measured configurations other than the headline serving run (``bench.py``).

    python -m mesh_b200.benchmarks cpu-tp2            # TinyLlama shape, cpu, TP=2 over loopback
    torchrun ... -m mesh_b200.benchmarks prefill      # 2k/8k/32k single-sequence prefill (TTFT)
    torchrun ... -m mesh_b200.benchmarks allreduce    # fused AR+norm vs NCCL vs host ring
    torchrun ... -m mesh_b200.benchmarks serve70b     # 70B TP=8, 256 sessions, 10% KV handoff
    torchrun ... -m mesh_b200.benchmarks gemmar       # decode GEMM + all-reduce: separate vs one launch

Every GPU number is timed with CUDA events on the launching stream after warm-up and reported as
the max over ranks; rank 0 prints one JSON line per measurement.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import time

import numpy as np


# ------------------------------------------------------------------------------------------ cpu TP=2
def _cpu_rank(rank, ports, out_q, prompt, gen, seed):
    from .config import get_preset
    from .models.sharding import shard_layout
    from .models.weights import synthetic_reference_weights
    from .oracle.tp_forward import ShardedForwardPass, shard_reference_weights
    from .parallel.tcp_plane import TensorPlane, WorkerRing
    cfg = get_preset("tinyllama-1.1b")
    plane = TensorPlane(port=ports[rank])
    addrs = [("127.0.0.1", p) for p in ports]
    w = synthetic_reference_weights(cfg, seed=seed)
    lay = shard_layout(cfg, rank, 2)
    fp = ShardedForwardPass(cfg, lay, shard_reference_weights(w, lay), WorkerRing(plane, rank, addrs, timeout_s=600))
    del w
    fp.ring.barrier()
    t0 = time.perf_counter()
    toks = fp.generate(prompt, gen)
    dt = time.perf_counter() - t0
    out_q.put((rank, toks, dt, fp.ring.time_ms, fp.ring.operations))
    fp.ring.barrier()
    plane.close()


def _free_ports(n):
    import socket
    socks, ports = [], []
    for _ in range(n):
        s = socket.socket()
        s.bind(("127.0.0.1", 0))
        socks.append(s)
        ports.append(s.getsockname()[1])
    for s in socks:
        s.close()
    return ports


def cpu_tp2(args):
    import multiprocessing as mp
    from .config import get_preset
    from .models.weights import synthetic_reference_weights
    from .oracle.forward import LocalForwardPass
    rng = np.random.default_rng(args.seed)
    cfg = get_preset("tinyllama-1.1b")
    prompt = rng.integers(0, cfg.vocab_size, 32).tolist()
    ctx = mp.get_context("spawn")
    oq = ctx.Queue()
    ports = _free_ports(2)
    ps = [ctx.Process(target=_cpu_rank, args=(r, ports, oq, prompt, args.gen, args.seed)) for r in range(2)]
    [p.start() for p in ps]
    res = sorted(oq.get(timeout=3600) for _ in range(2))
    [p.join() for p in ps]
    tp_dt = max(r[2] for r in res)
    w = synthetic_reference_weights(cfg, seed=args.seed)
    t0 = time.perf_counter()
    ref = LocalForwardPass(w).generate(prompt, args.gen)
    base_dt = time.perf_counter() - t0
    print(json.dumps({"config": "tinyllama-1.1b cpu tp2 loopback, prompt 32, greedy 16",
                      "tp2_tokens_per_s": args.gen / tp_dt, "tp2_seconds": tp_dt,
                      "allreduce_ms_per_rank": res[0][3], "allreduce_ops": res[0][4],
                      "oracle_tokens_per_s": args.gen / base_dt, "oracle_seconds": base_dt,
                      "tokens_match_oracle": res[0][1] == ref == res[1][1]}))


# ------------------------------------------------------------------------------------------ GPU helpers
def _dist():
    import torch
    import torch.distributed as dist
    from .parallel import dist as mdist
    di = mdist.init(timeout_s=300.0)
    return di, dist, torch


def _max_over_ranks(x, dist, torch, dev):
    t = torch.tensor([float(x)], dtype=torch.float64, device=dev)
    if dist.is_initialized():
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ------------------------------------------------------------------------------------ prefill sweep
def prefill(args):
    di, dist, torch = _dist()
    from .config import EngineConfig, get_preset
    from .models.llama import KVPool, LlamaRunner, StepMeta
    from .models.weights import synthetic_device_weights
    cfg = get_preset(args.model)
    dev = di.device
    maxlen = max(args.lengths)
    chunk = args.chunk
    w = synthetic_device_weights(cfg, di.rank, di.world, device=dev)
    pages = maxlen // 16 + 8
    kv = KVPool(cfg, w.layout.local_kv_heads, pages, 16, dev)
    ecfg = EngineConfig(max_seq_len=maxlen + 16, tp=di.world)
    runner = LlamaRunner(w, ecfg, kv, dev, group=dist.group.WORLD if di.world > 1 else None,
                         max_tokens=chunk, max_pos=maxlen + 16)
    bt = torch.arange(1, pages, device=dev, dtype=torch.int32)[None]
    g = torch.Generator().manual_seed(1)
    for L in args.lengths:
        ids_all = torch.randint(0, cfg.vocab_size, (L,), generator=g, dtype=torch.int32).to(dev)

        def run():
            nxt = None
            for a in range(0, L, chunk):
                b = min(L, a + chunk)
                pos = torch.arange(a, b, device=dev, dtype=torch.int32)
                m = StepMeta(ids=ids_all[a:b], pos=pos, slot=(bt[0, pos.long() // 16].long() * 16 + pos.long() % 16),
                             block_tables=bt, seq_lens=torch.tensor([b], device=dev, dtype=torch.int32),
                             cu_q=torch.tensor([0, b - a], device=dev, dtype=torch.int32),
                             last_idx=torch.tensor([b - a - 1], device=dev), max_q_len=b - a, decode=False)
                nxt = runner.forward(m)
            return nxt

        for _ in range(args.warmup):
            run()
        torch.cuda.synchronize()
        if di.world > 1:
            dist.barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(args.steps):
            run()
        e.record()
        torch.cuda.synchronize()
        ms = _max_over_ranks(s.elapsed_time(e) / args.steps, dist, torch, dev)
        flops = 2.0 * cfg.param_count() * L + 2.0 * cfg.num_layers * cfg.hidden_dim * L * L  # GEMMs + causal attn
        if di.rank == 0:
            print(json.dumps({"config": f"{args.model} prefill L={L} batch 1 tp{di.world}", "ttft_ms": ms,
                              "prefill_tokens_per_s": L / (ms / 1e3), "model_tflops": flops / (ms / 1e3) / 1e12,
                              "chunk_tokens": chunk}), flush=True)
    from .parallel import dist as mdist
    mdist.shutdown()


# ------------------------------------------------------------------------------------ prefill attention
def attnprefill(args):
    """Device time of causal paged prefill attention on one GPU for the shapes of one rank
    (Llama-3-8B heads at --tp): batches of sequences of one length, KV read in place from shuffled
    16-token pages. Kernels: the tcgen05 kernel ("tc"), the mma.sync kernel ("fa2") and, as a
    library reference, torch SDPA over the same K/V gathered into contiguous [S, H, L, D] (gather
    not timed). Reported as causal TFLOP/s (4 * L^2 / 2 * D per head) and its fraction of the
    measured bf16 peak."""
    import math
    import torch
    import torch.nn.functional as F
    from . import ops
    from .utils.opbench import peaks, timeit
    _, tf, src = peaks()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    hq, hkv, D, ps = 32 // args.tp, 8 // args.tp, 128, 16
    for spec in args.shapes:
        nseq, L = (int(x) for x in spec.split("x"))
        pp = (L + ps - 1) // ps
        npages = nseq * pp + 1
        kc = torch.randn(npages, hkv, ps, D, device=dev).to(torch.bfloat16)
        vc = torch.randn(npages, hkv, ps, D, device=dev).to(torch.bfloat16)
        bt = (torch.randperm(npages - 1, device=dev) + 1)[:nseq * pp].view(nseq, pp).int().contiguous()
        q = torch.randn(nseq * L, hq * D, device=dev).to(torch.bfloat16)
        out = torch.empty_like(q)
        cu = torch.arange(0, nseq + 1, device=dev, dtype=torch.int32) * L
        kl = torch.full((nseq,), L, dtype=torch.int32, device=dev)
        flops = 4.0 * nseq * hq * D * L * L / 2
        row = {"shape": f"{nseq}x{L} causal hq={hq} hkv={hkv} D={D}", "peak_source": src}
        iters = max(3, min(20, int(2e12 / flops)))
        for impl in args.impls:
            us = timeit(lambda i: ops.attn_prefill(q, kc, vc, cu, kl, bt, out, L, 1 / math.sqrt(D), impl=impl),
                        iters=iters)
            ops.scratch(dev).check(f"attn_prefill[{impl}]")
            row[f"{impl}_us"] = round(us, 1)
            row[f"{impl}_tflops"] = round(flops / us / 1e6, 1)
            row[f"{impl}_frac_of_measured_peak"] = round(flops / us / 1e6 / tf, 3)
        if not args.no_sdpa:
            kk = kc[bt.long()].permute(0, 2, 1, 3, 4).reshape(nseq, hkv, pp * ps, D)[:, :, :L]
            vv = vc[bt.long()].permute(0, 2, 1, 3, 4).reshape(nseq, hkv, pp * ps, D)[:, :, :L]
            kk = kk.repeat_interleave(hq // hkv, dim=1).contiguous()
            vv = vv.repeat_interleave(hq // hkv, dim=1).contiguous()
            qq = q.view(nseq, L, hq, D).transpose(1, 2).contiguous()
            us = timeit(lambda i: F.scaled_dot_product_attention(qq, kk, vv, is_causal=True), iters=iters)
            row["torch_sdpa_us"] = round(us, 1)
            row["torch_sdpa_tflops"] = round(flops / us / 1e6, 1)
            del kk, vv, qq
        print(json.dumps(row), flush=True)
        del kc, vc, q, out


# ------------------------------------------------------------------------------------ decode GEMM schedules
def decodemodes(args):
    """The four decode GEMMs of one TP rank (swap-AB, T tokens) under each schedule the tcgen05 GEMM
    has (0 = the planner's automatic choice, 1 = whole tiles, 2 = stream-K, 3 = cluster split-K),
    against cuBLAS on the same product; CUDA-graph timed with the weights rotated past L2. Shows
    whether the automatic choice is the fastest at a TP degree's shapes."""
    import torch
    from . import ops
    from .config import get_preset
    from .models.sharding import shard_layout
    from .models.weights import GU_BLOCK, pad_to
    from .utils.opbench import copies_for, timeit
    cfg = get_preset(args.model)
    lay = shard_layout(cfg, 0, args.tp)
    H, D, T = cfg.hidden_dim, cfg.head_dim, args.tokens
    i_loc = lay.mlp_cols
    shapes = {"qkv": ((lay.local_q_heads + 2 * lay.local_kv_heads) * D, H, ops.EPI_STORE_BF16),
              "o_proj": (H, lay.local_q_heads * D, ops.EPI_STORE_BF16),
              "gate_up": (2 * pad_to(i_loc, GU_BLOCK), H, ops.EPI_SILU_BF16),
              "down": (H, pad_to(i_loc, GU_BLOCK), ops.EPI_STORE_BF16)}
    dev = torch.device("cuda", 0)
    x_all = torch.randn(T, max(H, 8 * 4096), device=dev).to(torch.bfloat16)
    for name, (N, K, epi) in shapes.items():
        nc = min(copies_for(N * K * 2), 64)
        ws = [torch.randn(N, K, device=dev).mul_(0.02).to(torch.bfloat16) for _ in range(nc)]
        x = x_all[:, :K].contiguous()
        n_out = N // 2 if epi == ops.EPI_SILU_BF16 else N
        out = torch.empty(T, n_out, device=dev, dtype=torch.bfloat16)
        row = {"tp": args.tp, "op": name, "N": N, "K": K, "T": T,
               "plan": list(ops.ext().gemm_plan(N, T, K, epi, True, 0))}
        for mode in args.modes:
            try:
                row[f"mode{mode}_us"] = round(timeit(lambda i: ops.gemm(ws[i % nc], x, out, epi, trans=True, mode=mode)), 2)
            except RuntimeError as e:
                row[f"mode{mode}_us"] = f"n/a ({str(e)[:60]})"
        ref = torch.empty(T, N, device=dev, dtype=torch.bfloat16)
        row["cublas_us"] = round(timeit(lambda i: torch.mm(x, ws[i % nc].t(), out=ref)), 2)
        ops.scratch(dev).check("decodemodes")
        print(json.dumps(row), flush=True)
        del ws


# ------------------------------------------------------------------------------------ prefill GEMM kernels
def gemmcmp(args):
    """One prefill-sized product out = A @ B^T on one GPU: the SM-pair kernel, the one-SM kernel and
    cuBLAS (torch.mm), CUDA-graph timed with B rotated past L2, as TFLOP/s and fraction of the
    measured bf16 peak."""
    import torch
    from . import ops
    from .utils.opbench import copies_for, peaks, timeit
    _, tf, src = peaks()
    dev = torch.device("cuda", 0)
    M, N, K = args.M, args.N, args.K
    nc = min(copies_for(N * K * 2), 16)
    a = torch.randn(M, K, device=dev).to(torch.bfloat16)
    bs = [torch.randn(N, K, device=dev).mul_(0.02).to(torch.bfloat16) for _ in range(nc)]
    out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
    flops = 2.0 * M * N * K
    row = {"shape": f"M={M} N={N} K={K}", "peak_source": src}
    runs = {"pair": lambda i: ops.gemm_pair(a, bs[i % nc], out),
            "pair256": lambda i: ops.gemm_pair(a, bs[i % nc], out, tn=256),
            "pair128": lambda i: ops.gemm_pair(a, bs[i % nc], out, tn=128),
            "pair512": lambda i: ops.gemm_pair(a, bs[i % nc], out, tn=512),
            "one_sm": lambda i: ops.gemm(a, bs[i % nc], out, ops.EPI_STORE_BF16, trans=False),
            "cublas": lambda i: torch.mm(a, bs[i % nc].t(), out=out)}
    for name in args.impls:
        us = timeit(runs[name], iters=args.iters)
        row[f"{name}_us"] = round(us, 2)
        row[f"{name}_tflops"] = round(flops / us / 1e6, 1)
        row[f"{name}_frac"] = round(flops / us / 1e6 / tf, 3)
    ops.scratch(dev).check("gemmcmp")
    if args.trace:
        tr = torch.zeros(384, dtype=torch.int64, device=dev)
        ops.gemm_pair(a, bs[0], out, trace=tr)
        torch.cuda.synchronize()
        t = tr.cpu().double()
        t0 = t[t > 0].min()
        rel = lambda x: [round(float(v - t0) / 1e3, 2) if v > 0 else None for v in x]
        row["trace_leader_producer_us"] = rel(t[0:24])
        row["trace_peer_producer_us"] = rel(t[128:152])
        row["trace_mma_full_us"] = rel(t[256:280])
        d = (t[256 + 64] - t[256]) / 64 / 1e3 if t[256 + 64] > 0 else None
        row["trace_mma_us_per_kstep"] = round(float(d), 3) if d is not None else None
    print(json.dumps(row), flush=True)


# ------------------------------------------------------------------------------------ all-reduce sweep
def allreduce(args):
    """Per-call device time of the fused all-reduce + residual + RMSNorm (plain peer loads and NVLS
    multicast, one-shot and two-shot) against NCCL all-reduce + the same norm kernel, each captured
    in a CUDA graph of 20 calls (launch overhead excluded, as in the decode graphs) and reported as
    the max over ranks; plus the reference's host TCP ring for small sizes."""
    di, dist, torch = _dist()
    from . import ops
    from .parallel.symm import SymmWorkspace
    dev = di.device
    Hs = args.hidden
    Ts = args.tokens
    tmax = max(Ts)
    iters, reps = 20, 5
    results = []
    side = torch.cuda.Stream(dev)
    for H in Hs:
        ws = SymmWorkspace(tmax, H, dev)
        gamma = torch.ones(H, dtype=torch.bfloat16, device=dev)
        trace = torch.zeros(4, dtype=torch.int64, device=dev)
        for T in Ts:
            part = torch.randn(T, H, device=dev).to(torch.bfloat16)
            resid = torch.randn(T, H, device=dev).to(torch.bfloat16)
            nrm = torch.empty_like(resid)
            ws.partial(0, T).copy_(part)
            ws.partial(1, T).copy_(part)
            ws.resid(T).copy_(resid)

            def graphed(fn):
                for i in range(3):
                    fn(i)
                torch.cuda.synchronize()
                dist.barrier()
                g = torch.cuda.CUDAGraph()
                side.wait_stream(torch.cuda.current_stream())
                with torch.cuda.stream(side):
                    with torch.cuda.graph(g, stream=side):
                        for i in range(iters):
                            fn(i)
                torch.cuda.synchronize()
                dist.barrier()
                g.replay()
                g.replay()
                torch.cuda.synchronize()
                dist.barrier()
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record()
                for _ in range(reps):
                    g.replay()
                e.record()
                torch.cuda.synchronize()
                ops.scratch(dev).check("allreduce sweep")
                us = s.elapsed_time(e) * 1e3 / (reps * iters)
                del g
                return _max_over_ranks(us, dist, torch, dev)

            def phases(multicast, two_shot):
                for i in range(3):
                    ws.fused_allreduce_norm(T, i & 1, gamma, 1e-5, two_shot=two_shot, multicast=multicast)
                torch.cuda.synchronize()
                dist.barrier()
                ws.fused_allreduce_norm(T, 1, gamma, 1e-5, two_shot=two_shot, multicast=multicast, trace=trace)
                torch.cuda.synchronize()
                t = trace.tolist()
                return [round((t[1] - t[0]) / 1e3, 2), round((t[2] - t[1]) / 1e3, 2), round((t[3] - t[2]) / 1e3, 2)]

            row = {"T": T, "H": H, "world": di.world, "nvls": bool(ws.mc_base)}
            variants = [("p2p", False)] + ([("nvls", True)] if ws.mc_base else [])
            for name, mc in variants:
                for mode in ("oneshot", "twoshot"):
                    two = mode == "twoshot"
                    row[f"{name}_{mode}_us"] = graphed(
                        lambda i, m=mc, t2=two: ws.fused_allreduce_norm(T, i & 1, gamma, 1e-5, two_shot=t2,
                                                                         multicast=m))
                    row[f"{name}_{mode}_phases_us"] = phases(mc, two)
            row["barrier_us"] = graphed(lambda i: ws.barrier())
            buf = part.clone()
            r2 = resid.clone()
            row["nccl_plus_norm_us"] = graphed(
                lambda i: (dist.all_reduce(buf), ops.add_rmsnorm(r2, gamma, nrm, 1e-5, delta=buf)))
            if T * H <= 64 * 4096 and not args.no_host_ring:
                # the reference's algorithm: device -> host, ring over TCP, host -> device
                from .parallel.tcp_plane import TensorPlane, WorkerRing
                if not hasattr(allreduce, "_ring"):
                    plane = TensorPlane()
                    addrs = [None] * di.world
                    dist.all_gather_object(addrs, plane.addr)
                    allreduce._ring = WorkerRing(plane, di.rank, addrs)
                ring = allreduce._ring

                def host_ring_us():
                    dist.barrier()
                    torch.cuda.synchronize()
                    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    s.record()
                    for _ in range(5):
                        x = part.float().cpu().numpy()
                        y = ring.all_reduce(x)
                        torch.from_numpy(y).to(dev)
                    e.record()
                    torch.cuda.synchronize()
                    return _max_over_ranks(s.elapsed_time(e) * 1e3 / 5, dist, torch, dev)
                row["host_tcp_ring_us"] = host_ring_us()
            fused = {k: v for k, v in row.items() if k.endswith("shot_us")}
            best_k = min(fused, key=fused.get)
            best = fused[best_k]
            nbytes = 2 * T * H * 2 * (di.world - 1) / di.world  # ring-equivalent bytes per rank
            row["best"] = best_k
            row["fused_busbw_GBps"] = nbytes / (best * 1e-6) / 1e9
            row["speedup_vs_nccl"] = row["nccl_plus_norm_us"] / best
            results.append(row)
            if di.rank == 0:
                print(json.dumps(row), flush=True)
        del ws
    from .parallel import dist as mdist
    mdist.shutdown()


# ------------------------------------------------------------------------------------ GEMM + all-reduce
def gemmar(args):
    """Decode o_proj / down_proj followed by the TP all-reduce + residual + RMSNorm: per-call device
    time of (a) the GEMM alone, (b) the GEMM then the separate all-reduce kernel, (c) both in one
    launch (``gemm_allreduce_norm``), each captured in a CUDA graph of 20 calls with weights rotated
    past L2, max over ranks; plus the fused launch's per-phase timeline from %globaltimer stamps
    (medians over CTAs, us after the first CTA started)."""
    di, dist, torch = _dist()
    from . import ops
    from .config import get_preset
    from .models.sharding import shard_layout
    from .models.weights import GU_BLOCK, pad_to
    from .parallel.symm import SymmWorkspace
    cfg = get_preset(args.model)
    dev = di.device
    lay = shard_layout(cfg, di.rank, di.world)
    H = cfg.hidden_dim
    shapes = [("o_proj", lay.q_cols), ("down", pad_to(lay.mlp_cols, GU_BLOCK))]
    ws = SymmWorkspace(max(args.tokens), H, dev, multicast=not args.no_nvls)
    mc = bool(ws.mc_base) and di.world >= 8
    gamma = torch.ones(H, dtype=torch.bfloat16, device=dev)
    side = torch.cuda.Stream(dev)
    iters = 20

    def graphed(fn):
        for i in range(3):
            fn(i)
        torch.cuda.synchronize()
        ops.scratch(dev).check("gemmar warm-up")
        dist.barrier()
        g = torch.cuda.CUDAGraph()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            with torch.cuda.graph(g, stream=side):
                for i in range(iters):
                    fn(i)
        torch.cuda.synchronize()
        dist.barrier()
        g.replay()
        torch.cuda.synchronize()
        dist.barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(3):
            g.replay()
        e.record()
        torch.cuda.synchronize()
        ops.scratch(dev).check("gemmar")
        del g
        return round(_max_over_ranks(s.elapsed_time(e) * 1e3 / (3 * iters), dist, torch, dev), 2)

    for name, K in shapes:
        nc = max(2, min(32, (2 * 126 * 2 ** 20) // (H * K * 2) + 1))
        wts = [torch.randn(H, K, device=dev).mul_(0.02).to(torch.bfloat16) for _ in range(nc)]
        for T in args.tokens:
            x = torch.randn(T, K, device=dev).to(torch.bfloat16)
            ws.resid(T).normal_()
            row = {"op": name, "T": T, "K": K, "H": H, "world": di.world, "nvls": mc}
            row["gemm_us"] = graphed(lambda i: ops.linear(x, wts[i % nc], out=ws.partial(i & 1, T)))
            two = T * H * 2 * (di.world - 1) > (8 << 20) and di.world > 2
            row["gemm_then_ar_us"] = graphed(lambda i: (
                ops.linear(x, wts[i % nc], out=ws.partial(i & 1, T)),
                ws.fused_allreduce_norm(T, i & 1, gamma, 1e-5, two_shot=two, multicast=mc)))
            row["fused_us"] = graphed(lambda i: ws.gemm_allreduce_norm(x, wts[i % nc], i & 1, gamma, 1e-5,
                                                                       multicast=mc))
            plan = ops.ext().gemm_plan(H, T, K, ops.EPI_STORE_BF16, True, dev.index)
            tr = torch.zeros(160 * 32, dtype=torch.int64, device=dev)
            dist.barrier()
            ws.gemm_allreduce_norm(x, wts[0], 0, gamma, 1e-5, multicast=mc, trace=tr)
            torch.cuda.synchronize()
            t = tr.view(-1, 32)[: plan[4]].cpu()
            t0 = int(t[:, 0].min())
            rel = lambda c, sel=None: ((t[:, c] if sel is None else t[sel, c]).double() - t0) / 1e3  # noqa: E731
            med = lambda v: round(float(v.median()), 2) if len(v) else None  # noqa: E731
            red = t[:, 18] > 0
            row["plan"] = {"bn": plan[0], "grid": plan[4], "ck": plan[7], "dp_tiles": plan[5]}
            row["timeline_us"] = {
                "cta_start_max": round(float(rel(0).max()), 2), "griddep_passed": med(rel(1)),
                "mma_done_max": round(float(rel(4).max()), 2), "tail_start_med": med(rel(16)),
                "tail_start_max": round(float(rel(16).max()), 2), "phase0_arrived_max": round(float(rel(17).max()), 2),
                "reducers": int(red.sum()), "phase0_passed_med": med(rel(18, red)), "rows_done_med": med(rel(19, red)),
                "phase1_arrived_max": round(float(rel(20, red).max()), 2) if red.any() else None,
                "phase1_passed_cta0": round(float(rel(21)[0]), 2), "exit_max": round(float(rel(7).max()), 2)}
            if di.rank == 0:
                print(json.dumps(row), flush=True)
        del wts
    del ws
    from .parallel import dist as mdist
    mdist.shutdown()


# ------------------------------------------------------------------------------------ 70B serving
def serve70b(args):
    """256 sessions, prompts U[128,2048], 256 output tokens, served by decode queue A; after half
    the decode steps 10% of the sessions are handed off to a second decode queue B (its own engine,
    KV pool and CUDA graphs over the same weights): each session's pages are gathered on the device,
    re-allocated in B's pool and scattered there, and both queues keep decoding to the end."""
    di, dist, torch = _dist()
    from .config import EngineConfig, get_preset
    from .engine.serving import Engine
    from .models.llama import KVPool, LlamaRunner
    from .models.weights import synthetic_device_weights
    cfg = get_preset(args.model)
    if args.layers:
        cfg = cfg.replace(num_layers=args.layers)
    dev = di.device
    S, G = args.sessions, args.gen
    rng = np.random.default_rng(7)
    lens = rng.integers(128, 2049, S).tolist()
    maxs = (2048 + G + 15) // 16 * 16
    ecfg = EngineConfig(tp=di.world, max_seq_len=maxs, prefill_chunk_tokens=args.chunk)
    w = synthetic_device_weights(cfg, di.rank, di.world, device=dev)
    group = dist.group.WORLD if di.world > 1 else None
    pages = sum((l + G + 15) // 16 for l in lens) + 64
    eng = Engine(LlamaRunner(w, ecfg, KVPool(cfg, w.layout.local_kv_heads, pages, 16, dev), dev, group=group,
                             max_tokens=args.chunk + 2048), ecfg, max_batch=S)
    n_hand = max(1, int(args.handoff * S)) if args.handoff > 0 else 0
    eng_b = None
    if n_hand:
        pages_b = sum((l + G + 15) // 16 for l in lens[:n_hand]) + 16
        eng_b = Engine(LlamaRunner(w, ecfg, KVPool(cfg, w.layout.local_kv_heads, pages_b, 16, dev), dev, group=group,
                                   max_tokens=max(n_hand, 64)), ecfg, max_batch=n_hand)
    prompts = [rng.integers(0, cfg.vocab_size, l).tolist() for l in lens]
    ev0, evp, evd = (torch.cuda.Event(enable_timing=True) for _ in range(3))
    ev0.record()
    sids = [eng.submit(p, G) for p in prompts]
    while eng.waiting:
        eng.prefill_step()
    evp.record()
    steps = 0
    handed = 0
    hand_ms = 0.0
    while eng.has_work() or (eng_b is not None and eng_b.has_work()):
        if eng.has_work():
            eng.decode_step()
        if eng_b is not None and eng_b.has_work():
            eng_b.decode_step()
        steps += 1
        if steps == G // 2 and n_hand:
            h0, h1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            h0.record()
            for sid in sids[:n_hand]:
                if eng.sessions[sid].status != "decoding":
                    continue
                eng_b.import_session(eng.export_session(sid))
                handed += 1
            h1.record()
            torch.cuda.synchronize()
            hand_ms = h0.elapsed_time(h1)
    evd.record()
    eng.flush_history()
    if eng_b is not None:
        eng_b.flush_history()
    torch.cuda.synchronize()
    dec_ms = _max_over_ranks(evp.elapsed_time(evd), dist, torch, dev)
    pre_ms = _max_over_ranks(ev0.elapsed_time(evp), dist, torch, dev)
    hand_ms = _max_over_ranks(hand_ms, dist, torch, dev)
    ttft = sorted(ev0.elapsed_time(eng.sessions[s].ttft_event) for s in sids if s in eng.sessions)
    p50 = _max_over_ranks(ttft[len(ttft) // 2], dist, torch, dev)
    if di.rank == 0:
        print(json.dumps({"config": f"{cfg.name} tp{di.world} {S} sessions U[128,2048] x {G}",
                          "decode_tokens_per_s": S * (G - 1) / (dec_ms / 1e3), "p50_ttft_ms": p50,
                          "prefill_ms": pre_ms, "decode_ms": dec_ms, "sessions_handed_off": handed,
                          "handoff_ms": hand_ms, "layers": cfg.num_layers}), flush=True)
    eng.close()
    if eng_b is not None:
        eng_b.close()
    from .parallel import dist as mdist
    mdist.shutdown()


def main():
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="cmd", required=True)
    c1 = sub.add_parser("cpu-tp2")
    c1.add_argument("--gen", type=int, default=16)
    c1.add_argument("--seed", type=int, default=0)
    c3 = sub.add_parser("prefill")
    c3.add_argument("--model", default="llama3-8b")
    c3.add_argument("--lengths", type=int, nargs="+", default=[2048, 8192, 32768])
    c3.add_argument("--chunk", type=int, default=8192)
    c3.add_argument("--steps", type=int, default=3)
    c3.add_argument("--warmup", type=int, default=2)
    c7 = sub.add_parser("attnprefill")
    c7.add_argument("--shapes", nargs="+", default=["8x512", "64x512", "1x2048", "1x8192", "1x32768"])
    c7.add_argument("--tp", type=int, default=1)
    c7.add_argument("--impls", nargs="+", default=["tc", "fa2"])
    c7.add_argument("--no-sdpa", action="store_true")
    c9 = sub.add_parser("decodemodes")
    c9.add_argument("--model", default="llama3-8b")
    c9.add_argument("--tp", type=int, default=8)
    c9.add_argument("--tokens", type=int, default=64)
    c9.add_argument("--modes", type=int, nargs="+", default=[0, 1, 2, 3])
    c8 = sub.add_parser("gemmcmp")
    c8.add_argument("--M", type=int, default=4096)
    c8.add_argument("--N", type=int, default=4096)
    c8.add_argument("--K", type=int, default=4096)
    c8.add_argument("--iters", type=int, default=20)
    c8.add_argument("--impls", nargs="+", default=["pair", "one_sm", "cublas"])
    c8.add_argument("--trace", action="store_true")
    c5 = sub.add_parser("allreduce")
    c5.add_argument("--tokens", type=int, nargs="+", default=[1, 8, 64, 512, 4096, 8192])
    c5.add_argument("--hidden", type=int, nargs="+", default=[4096, 8192])
    c5.add_argument("--no-host-ring", action="store_true")
    c6 = sub.add_parser("gemmar")
    c6.add_argument("--model", default="llama3-8b")
    c6.add_argument("--tokens", type=int, nargs="+", default=[1, 8, 64, 128])
    c6.add_argument("--no-nvls", action="store_true")
    c4 = sub.add_parser("serve70b")
    c4.add_argument("--model", default="llama3-70b")
    c4.add_argument("--sessions", type=int, default=256)
    c4.add_argument("--gen", type=int, default=256)
    c4.add_argument("--chunk", type=int, default=8192)
    c4.add_argument("--handoff", type=float, default=0.1)
    c4.add_argument("--layers", type=int, default=0)
    a = ap.parse_args()
    {"cpu-tp2": cpu_tp2, "prefill": prefill, "allreduce": allreduce, "serve70b": serve70b,
     "gemmar": gemmar, "attnprefill": attnprefill, "gemmcmp": gemmcmp, "decodemodes": decodemodes}[a.cmd](a)


if __name__ == "__main__":
    main()
