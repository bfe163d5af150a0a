"""Tensor-parallel paths on 2, 4 and 8 GPUs, run as
spawned child processes (NCCL for plumbing with its NVLS off; the fused kernels on plain peer loads,
except the tests that check their NVLS multicast path).

* the fused peer-memory all-reduce + residual + RMSNorm kernel (one-shot and two-shot) against an
  fp32 reference built from NCCL all-gathered partials;
* the decode GEMM with the all-reduce, residual add, RMSNorm and all-gather in the same launch, for
  every GEMM schedule, against the same reference;
* the bounded-wait error path: a rank that never joins makes the other's wait run out, the kernel
  returns ERR_PEER_TIMEOUT within the limit, and a collective reset makes the workspace usable;
* the TP=N decoder's prefill and decode logits against TP=1.
A test needing more GPUs than the machine has is skipped.
"""
import os
import socket
import tempfile
import traceback

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _run(fn, world, *args):
    import torch.multiprocessing as mp
    port = _free_port()
    with tempfile.TemporaryDirectory() as d:
        crash = None
        try:
            mp.spawn(_entry, args=(world, port, fn, d, args), nprocs=world, join=True)
        except mp.ProcessExitedException as e:  # report the ranks' own errors, if any, with the crash
            crash = str(e)
        errs, skips = [], []
        for r in range(world):
            f = os.path.join(d, f"err{r}")
            if os.path.exists(f):
                errs.append(open(f).read())
            f = os.path.join(d, f"skip{r}")
            if os.path.exists(f):
                skips.append(open(f).read())
        assert not errs and crash is None, "\n".join(errs + ([crash] if crash else []))
        if skips:
            pytest.skip(skips[0])


def _entry(rank, world, port, fn, d, args):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    # rendezvous through a file in the test's private directory: no TCP port to race for
    dist.init_process_group("nccl", init_method=f"file://{os.path.join(d, 'pg_store')}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        reason = fn(rank, world, *args)
        if isinstance(reason, str):
            with open(os.path.join(d, f"skip{rank}"), "w") as f:
                f.write(reason)
    except Exception:
        with open(os.path.join(d, f"err{rank}"), "w") as f:
            f.write(f"rank {rank}:\n" + traceback.format_exc())
    finally:
        try:
            torch.cuda.synchronize()
            dist.barrier()
        except Exception:
            pass
        dist.destroy_process_group()


def _ar_check(rank, world, multicast=False):
    import torch.distributed as dist
    from mesh_b200 import ops
    from mesh_b200.models.sharding import even_split
    from mesh_b200.ops import reference as ref
    from mesh_b200.parallel.symm import SymmWorkspace
    dev = torch.device("cuda", rank)
    H = 4096
    ws = SymmWorkspace(1024, H, dev, multicast=multicast)
    if multicast and not ws.mc_base:
        return "symmetric memory has no NVLS multicast mapping on this node"
    gamma = (1 + 0.1 * torch.randn(H, generator=torch.Generator().manual_seed(1))).to(torch.bfloat16).to(dev)
    parity = 0
    for T in (1, 7, 64, 300, 1024):
        for two_shot in (False, True):
            resid0 = torch.randn(T, H, generator=torch.Generator().manual_seed(T)).to(torch.bfloat16).to(dev)
            part = torch.randn(T, H, generator=torch.Generator().manual_seed(100 * T + rank)).to(torch.bfloat16).to(dev)
            ws.resid(T).copy_(resid0)
            ws.partial(parity, T).copy_(part)
            ws.fused_allreduce_norm(T, parity, gamma, 1e-5, two_shot=two_shot, timeout_s=5.0, multicast=multicast)
            torch.cuda.synchronize()
            ops.scratch(dev).check("ar")
            allp = torch.empty(world, T, H, dtype=torch.bfloat16, device=dev)
            dist.all_gather_into_tensor(allp.view(-1), part.view(-1))
            want_r = (resid0.float() + allp.float().sum(0)).to(torch.bfloat16)
            want_n = ref.rmsnorm(want_r.float(), gamma, 1e-5)
            got_r, got_n = ws.resid(T), ws.normed(T)
            # two-shot leaves each residual row with the rank that reduced it
            r0, nr = even_split(T, world, rank) if two_shot else (0, T)
            got_r, want_own = got_r[r0:r0 + nr].float(), want_r[r0:r0 + nr].float()
            er = ((got_r - want_own).norm() / want_own.norm()).item() if nr else 0.0
            en = ((got_n.float() - want_n).norm() / want_n.norm()).item()
            assert er < 1e-2 and en < 1e-2, (T, two_shot, er, en)
            parity ^= 1


def _push_check(rank, world):
    """Fused GEMM -> reduce-scatter: every rank's GEMM epilogue pushes its partial rows to the owner
    ranks over NVLink, then the owners reduce locally, add the residual, normalise and all-gather."""
    import torch.distributed as dist
    from mesh_b200 import ops
    from mesh_b200.models.sharding import even_split
    from mesh_b200.ops import reference as ref
    from mesh_b200.parallel.symm import SymmWorkspace
    dev = torch.device("cuda", rank)
    H, K = 2048, 1024
    ws = SymmWorkspace(512, H, dev)
    gamma = torch.ones(H, dtype=torch.bfloat16, device=dev)
    w = (torch.randn(H, K, generator=torch.Generator().manual_seed(50 + rank)) * 0.05).to(torch.bfloat16).to(dev)
    parity = 0
    for T, two_shot in ((64, True), (1, False), (300, True), (5, False)):
        x = torch.randn(T, K, generator=torch.Generator().manual_seed(T + 7 * rank)).to(torch.bfloat16).to(dev)
        resid0 = torch.randn(T, H, generator=torch.Generator().manual_seed(T)).to(torch.bfloat16).to(dev)
        ws.resid(T).copy_(resid0)
        ops.linear(x, w, out=torch.empty(T, H, dtype=torch.bfloat16, device=dev),
                   push=ws.push_args(T, parity, two_shot))
        ws.push_reduce_norm(T, parity, gamma, 1e-5, two_shot=two_shot)
        torch.cuda.synchronize()
        ops.scratch(dev).check("push")
        part = (x.float() @ w.float().T).to(torch.bfloat16)
        allp = torch.empty(world, T, H, dtype=torch.bfloat16, device=dev)
        dist.all_gather_into_tensor(allp.view(-1), part.contiguous().view(-1))
        want_r = (resid0.float() + allp.float().sum(0))
        r0, nr = even_split(T, world, rank) if two_shot else (0, T)
        got = ws.resid(T).float()[r0:r0 + nr]
        e = ((got - want_r[r0:r0 + nr]).norm() / want_r[r0:r0 + nr].norm()).item() if nr else 0.0
        en = ((ws.normed(T).float() - ref.rmsnorm(want_r.to(torch.bfloat16).float(), gamma, 1e-5)).norm() /
              want_r.norm()).item()
        assert e < 2e-2 and en < 2e-2, (T, two_shot, e, en)
        parity ^= 1


def _gemm_ar_check(rank, world, multicast=False):
    """Decode o_proj/down GEMM with the all-reduce, residual add and RMSNorm in its own launch: the
    owned residual rows and every normed row against fp32 sums of NCCL all-gathered partials, for
    the automatic schedule and each forced one (whole tiles, stream-K, cluster split-K), several
    launches in a row over alternating push slots."""
    import torch.distributed as dist
    from mesh_b200 import ops
    from mesh_b200.models.sharding import even_split
    from mesh_b200.ops import reference as ref
    from mesh_b200.parallel.symm import SymmWorkspace
    dev = torch.device("cuda", rank)
    H = 4096
    ws = SymmWorkspace(256, H, dev, multicast=multicast)
    if multicast and not ws.mc_base:
        return "symmetric memory has no NVLS multicast mapping on this node"
    gamma = (1 + 0.1 * torch.randn(H, generator=torch.Generator().manual_seed(3))).to(torch.bfloat16).to(dev)
    parity = 0
    cases = [(512, 64, 0), (2048, 64, 0), (1792, 64, 0), (512, 1, 0), (2048, 5, 0), (1024, 256, 0),
             (1024, 64, 1), (2048, 64, 2), (2048, 64, 3), (2048, 16, 3)]
    for i, (K, T, mode) in enumerate(cases):
        g = torch.Generator().manual_seed(1000 * i + rank)
        w = (torch.randn(H, K, generator=g) * 0.03).to(torch.bfloat16).to(dev)
        x = torch.randn(T, K, generator=g).to(torch.bfloat16).to(dev)
        resid0 = torch.randn(T, H, generator=torch.Generator().manual_seed(77 + i)).to(torch.bfloat16).to(dev)
        for rep in range(2):  # back-to-back launches: epochs, counters and both push slots are reused
            ws.resid(T).copy_(resid0)
            ws.normed(T).fill_(float("nan"))
            torch.cuda.synchronize()
            dist.barrier()
            ws.gemm_allreduce_norm(x, w, parity, gamma, 1e-5, timeout_s=5.0, mode=mode, multicast=multicast)
            torch.cuda.synchronize()
            ops.scratch(dev).check(f"gemm_ar K={K} T={T} mode={mode}")
            part = (x.float() @ w.float().T).to(torch.bfloat16)
            allp = torch.empty(world, T, H, dtype=torch.bfloat16, device=dev)
            dist.all_gather_into_tensor(allp.view(-1), part.contiguous().view(-1))
            want_r = (resid0.float() + allp.float().sum(0)).to(torch.bfloat16)
            want_n = ref.rmsnorm(want_r.float(), gamma, 1e-5)
            r0, nr = even_split(T, world, rank)
            if nr:
                got_r = ws.resid(T)[r0:r0 + nr].float()
                er = ((got_r - want_r[r0:r0 + nr].float()).norm() / want_r[r0:r0 + nr].float().norm()).item()
                assert er < 1e-2, (K, T, mode, rep, "resid", er)
            got_n = ws.normed(T).float()
            assert torch.isfinite(got_n).all(), (K, T, mode, rep, "normed rows not written")
            en = ((got_n - want_n).norm() / want_n.norm()).item()
            assert en < 2e-2, (K, T, mode, rep, "normed", en)
            parity ^= 1


def _timeout_check(rank, world):
    import time
    import torch.distributed as dist
    from mesh_b200 import ops
    from mesh_b200.parallel.symm import SymmWorkspace
    dev = torch.device("cuda", rank)
    H = 1024
    ws = SymmWorkspace(64, H, dev, multicast=False)  # fault-path tests use plain peer loads only
    gamma = torch.ones(H, dtype=torch.bfloat16, device=dev)
    dist.barrier()
    if rank == 0:
        # the peer never joins this collective: the bounded wait must give up and report
        t0 = time.time()
        ws.fused_allreduce_norm(8, 0, gamma, 1e-5, two_shot=False, timeout_s=0.5)
        torch.cuda.synchronize()
        dt = time.time() - t0
        code = int(ops.scratch(dev).err.item())
        assert code == 4, f"expected ERR_PEER_TIMEOUT, got {code}"
        assert dt < 10.0, dt
    dist.barrier()
    ws.reset()
    # after the reset a normal collective works again
    ws.resid(8).zero_()
    ws.partial(0, 8).fill_(1.0)
    ws.fused_allreduce_norm(8, 0, gamma, 1e-5, two_shot=False, timeout_s=5.0)
    torch.cuda.synchronize()
    ops.scratch(dev).check("ar after reset")
    assert torch.allclose(ws.resid(8).float(), torch.full((8, H), float(world), device=dev))


def _tp_logits(rank, world, preset="small", layers=0, nvls=False, ar="auto"):
    """Prefill of one prompt, then decode steps of a 3-session batch (with ar="gemm_ar" the decode
    steps run the all-reduce inside the GEMM launch), teacher-forced with the TP=1 run's greedy
    tokens: every step's full-vocabulary logits at TP=world against TP=1, and each TP=world token
    equal to the argmax of its own logits."""
    import torch.distributed as dist
    from mesh_b200.config import EngineConfig, get_preset
    from mesh_b200.models.llama import KVPool, LlamaRunner, StepMeta
    from mesh_b200.models.sharding import even_split
    from mesh_b200.models.weights import synthetic_device_weights
    dev = torch.device("cuda", rank)
    cfg = get_preset(preset)
    if layers:
        cfg = cfg.replace(num_layers=layers)
    if cfg.num_kv_heads % world:
        return f"{preset} has {cfg.num_kv_heads} KV heads, not divisible over {world} ranks"
    ecfg = EngineConfig(max_seq_len=256, nvls=nvls, allreduce_impl=ar)
    gen = torch.Generator().manual_seed(5)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=gen).tolist() for n in (40, 17, 33)]
    steps = 4

    def run(world_, rank_, group, forced=None):
        w = synthetic_device_weights(cfg, rank_, world_, seed=9, device=dev, norm_noise=True)
        kv = KVPool(cfg, w.layout.local_kv_heads, 64, 16, dev)
        r = LlamaRunner(w, ecfg, kv, dev, group=group, max_tokens=256)
        r.keep_logits = True
        B = len(prompts)
        bt = torch.zeros(B, 8, dtype=torch.int32, device=dev)
        for b in range(B):
            bt[b, :4] = torch.arange(1 + 4 * b, 5 + 4 * b)
        logits, toks, nxt = [], [], []
        for b, p in enumerate(prompts):
            T = len(p)
            pos = torch.arange(T, device=dev)
            m = StepMeta(ids=torch.tensor(p, dtype=torch.int32, device=dev), pos=pos.int(),
                         slot=(bt[b, pos // 16].long() * 16 + pos % 16), block_tables=bt[b:b + 1],
                         seq_lens=torch.tensor([T], dtype=torch.int32, device=dev),
                         cu_q=torch.tensor([0, T], dtype=torch.int32, device=dev),
                         last_idx=torch.tensor([T - 1], device=dev), max_q_len=T, decode=False)
            ids = r.forward(m)
            logits.append(r.last_logits[0].float().clone())
            nxt.append(int(ids[0]))
        toks.append(list(nxt))
        for st in range(steps):
            feed = forced[st] if forced is not None else nxt
            lens = [len(p) + st for p in prompts]
            pos = torch.tensor(lens, device=dev)
            m = StepMeta(ids=torch.tensor(feed, dtype=torch.int32, device=dev), pos=pos.int(),
                         slot=(bt[torch.arange(B, device=dev), pos // 16].long() * 16 + pos % 16),
                         block_tables=bt, seq_lens=(pos + 1).int(), max_q_len=128, decode=True)
            ids = r.forward(m)
            for b in range(B):
                logits.append(r.last_logits[b].float().clone())
            nxt = ids.tolist()
            toks.append(list(nxt))
        torch.cuda.synchronize()
        return logits, toks

    full, toks1 = run(1, 0, None)
    part, toksn = run(world, rank, dist.group.WORLD, forced=toks1)
    sizes = [even_split(cfg.vocab_size, world, r)[1] for r in range(world)]
    for i, (f, p) in enumerate(zip(full, part)):
        parts = [torch.empty(n, device=dev) for n in sizes]
        dist.all_gather(parts, p.contiguous())
        tp = torch.cat(parts)
        err = ((tp - f).norm() / f.norm()).item()
        assert err < 3e-2, (i, err)
        step, b = (0, i) if i < len(prompts) else (1 + (i - len(prompts)) // len(prompts), (i - len(prompts)) % 3)
        assert toksn[step][b] == int(tp.argmax()), (i, toksn[step][b], int(tp.argmax()))


def _embed_check(rank, world):
    """Vocabulary-parallel embedding: every token's row comes from the rank that owns it (peer loads),
    against a lookup in the full table plus the fp32 RMSNorm."""
    from mesh_b200 import ops
    from mesh_b200.models.sharding import even_split
    from mesh_b200.ops import reference as ref
    from mesh_b200.parallel.symm import SymmTable
    dev = torch.device("cuda", rank)
    V, H = 1003, 4096
    full = torch.randn(V, H, generator=torch.Generator().manual_seed(11)).to(torch.bfloat16).to(dev)
    v0, vn = even_split(V, world, rank)
    table = SymmTable(full[v0:v0 + vn].contiguous(), V)
    gamma = (1 + 0.1 * torch.randn(H, generator=torch.Generator().manual_seed(12))).to(torch.bfloat16).to(dev)
    ids = torch.randint(0, V, (97,), generator=torch.Generator().manual_seed(13)).int().to(dev)
    ids[:world] = torch.tensor([even_split(V, world, r)[0] for r in range(world)], device=dev)  # every owner
    resid = torch.full((97, H), float("nan"), dtype=torch.bfloat16, device=dev)
    normed = torch.full_like(resid, float("nan"))
    ops.embed_peer_norm(table.bases, ids, V, gamma, 1e-5, resid, normed)
    torch.cuda.synchronize()
    ops.scratch(dev).check("embed_peer_norm")
    want = full[ids.long()]
    assert torch.equal(resid, want)
    wn = ref.rmsnorm(want.float(), gamma, 1e-5)
    assert ((normed.float() - wn).norm() / wn.norm()).item() < 1e-2


@pytest.mark.parametrize("world", [2, 4, 8])
def test_vocab_parallel_embedding(world):
    _need(world)
    _run(_embed_check, world)


def _stall_check(rank, world):
    """Failure detection through the engine: rank 1 stalls on the host between two decode steps for
    longer than the collectives' bound (0.5 s, NVLS off), rank 0's all-reduce waits run out, and
    rank 0's engine raises a clean RuntimeError when it reads the step back; after a collective
    reset of the workspace both engines step again without error."""
    import time
    import torch.distributed as dist
    from mesh_b200.config import EngineConfig, get_preset
    from mesh_b200.engine.serving import Engine
    from mesh_b200.models.llama import KVPool, LlamaRunner
    from mesh_b200.models.weights import synthetic_device_weights
    dev = torch.device("cuda", rank)
    cfg = get_preset("small")
    ecfg = EngineConfig(max_seq_len=256, nvls=False, allreduce_timeout_s=0.5, tp=world)
    w = synthetic_device_weights(cfg, rank, world, seed=3, device=dev)
    kv = KVPool(cfg, w.layout.local_kv_heads, 64, 16, dev)
    eng = Engine(LlamaRunner(w, ecfg, kv, dev, group=dist.group.WORLD, max_tokens=256), ecfg, max_batch=4)
    g = torch.Generator().manual_seed(8)
    for n in (11, 23):
        eng.submit(torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist(), 12)
    while eng.waiting:
        eng.prefill_step()
    for _ in range(2):
        eng.decode_step()
    eng.flush_history()
    dist.barrier()
    if rank == 1:
        time.sleep(1.5)  # between steps: nothing of this rank is in flight
    eng.decode_step()
    raised = False
    try:
        eng.flush_history()
    except RuntimeError as e:
        raised = "peer timeout" in str(e) or "device error code 4" in str(e)
    flags = torch.tensor([1 if raised else 0], device=dev)
    dist.all_reduce(flags)
    if rank == 0:
        assert raised, "rank 0's bounded waits must have run out and surfaced as an exception"
    eng.runner.symm.reset()
    eng.decode_step()
    eng.flush_history()  # no error after the reset
    eng.close()


def test_engine_surfaces_peer_stall_2gpu():
    _need(2)
    _run(_stall_check, 2)


def _need(n):
    if torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPUs")


@pytest.mark.parametrize("world", [2, 4, 8])
def test_fused_allreduce_norm(world):
    _need(world)
    _run(_ar_check, world)


@pytest.mark.parametrize("world", [2, 8])
def test_fused_allreduce_norm_nvls(world):
    _need(world)
    _run(_ar_check, world, True)


def test_fused_gemm_reduce_scatter_push_2gpu():
    _need(2)
    _run(_push_check, 2)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_gemm_allreduce_norm_one_launch(world):
    _need(world)
    _run(_gemm_ar_check, world)


@pytest.mark.parametrize("world", [2, 8])
def test_gemm_allreduce_norm_one_launch_nvls(world):
    _need(world)
    _run(_gemm_ar_check, world, True)


def test_allreduce_bounded_wait_reports_timeout_2gpu():
    _need(2)
    _run(_timeout_check, 2)


def _overlap_check(rank, world):
    """Prefill chunks of several prompts run as two overlapped halves (two streams, two symmetric
    workspaces) and as one piece: the generated tokens are bitwise the same, and halves ran."""
    import torch.distributed as dist
    from mesh_b200 import ops
    from mesh_b200.config import EngineConfig, get_preset
    from mesh_b200.engine.serving import Engine
    from mesh_b200.models.llama import KVPool, LlamaRunner
    from mesh_b200.models.weights import synthetic_device_weights
    dev = torch.device("cuda", rank)
    cfg = get_preset("small")
    gen = torch.Generator().manual_seed(11)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=gen).tolist() for n in (300, 280, 310, 290, 130)]
    out = {}
    for overlap in (False, True):
        ecfg = EngineConfig(max_seq_len=512, prefill_chunk_tokens=2048, prefill_overlap=overlap, tp=world)
        w = synthetic_device_weights(cfg, rank, world, seed=21, device=dev, norm_noise=True)
        kv = KVPool(cfg, w.layout.local_kv_heads, 256, 16, dev)
        r = LlamaRunner(w, ecfg, kv, dev, group=dist.group.WORLD, max_tokens=2048)
        eng = Engine(r, ecfg, max_batch=8)
        out[overlap] = eng.generate(prompts, 6)
        torch.cuda.synchronize()
        ops.scratch(dev).check("overlap")
        assert r.overlap_prefill == overlap and (r.split_steps > 0) == overlap, (overlap, r.split_steps)
        eng.close()
    assert out[True] == out[False]


def test_prefill_overlap_halves_equal_whole_2gpu():
    _need(2)
    _run(_overlap_check, 2)


@pytest.mark.parametrize("ar", ["auto", "gemm_ar"])
def test_tp2_logits_match_tp1(ar):
    _need(2)
    _run(_tp_logits, 2, "small", 0, False, ar)


@pytest.mark.parametrize("world", [4, 8])
def test_tpn_llama3_shape_logits_match_tp1(world):
    """Llama-3-8B-shaped (2 layers) at TP=4/8, NVLS on at 8 ranks as in serving."""
    _need(world)
    _run(_tp_logits, world, "llama3-8b", 2, world >= 8, "gemm_ar")
