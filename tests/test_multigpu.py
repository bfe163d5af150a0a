"""Tensor-parallel paths on 2 GPUs, run as spawned child processes (NCCL for plumbing with its NVLS
off; the fused kernels on plain peer loads, except the test that checks their NVLS multicast path).

* the fused peer-memory all-reduce + residual + RMSNorm kernel (one-shot and two-shot) against an
  fp32 reference built from NCCL all-gathered partials;
* the bounded-wait error path: a rank that never joins makes the other's wait run out, the kernel
  returns ERR_PEER_TIMEOUT within the limit, and a collective reset makes the workspace usable;
* the TP=2 decoder's logits against TP=1.
"""
import os
import socket
import tempfile
import traceback

import pytest
import torch

pytestmark = pytest.mark.gpu

NEED = 2


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
        mp.spawn(_entry, args=(world, port, fn, d, args), nprocs=world, join=True)
        errs, skips = [], []
        for r in range(world):
            f = os.path.join(d, f"err{r}")
            if os.path.exists(f):
                errs.append(open(f).read())
            f = os.path.join(d, f"skip{r}")
            if os.path.exists(f):
                skips.append(open(f).read())
        assert not errs, "\n".join(errs)
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
            er = ((got_r.float() - want_r.float()).norm() / want_r.float().norm()).item()
            en = ((got_n.float() - want_n).norm() / want_n.norm()).item()
            assert er < 1e-2 and en < 1e-2, (T, two_shot, er, en)
            parity ^= 1


def _push_check(rank, world):
    """Fused GEMM -> reduce-scatter: every rank's GEMM epilogue pushes its partial rows to the owner
    ranks over NVLink, then the owners reduce locally, add the residual, normalise and all-gather."""
    import torch.distributed as dist
    from mesh_b200 import ops
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
        got = ws.resid(T).float()
        e = ((got - want_r).norm() / want_r.norm()).item()
        en = ((ws.normed(T).float() - ref.rmsnorm(want_r.to(torch.bfloat16).float(), gamma, 1e-5)).norm() /
              want_r.norm()).item()
        assert e < 2e-2 and en < 2e-2, (T, two_shot, e, en)
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


def _tp_logits(rank, world):
    import torch.distributed as dist
    from mesh_b200.config import EngineConfig, get_preset
    from mesh_b200.models.llama import KVPool, LlamaRunner, StepMeta
    from mesh_b200.models.weights import synthetic_device_weights
    dev = torch.device("cuda", rank)
    cfg = get_preset("small")
    ecfg = EngineConfig(max_seq_len=256)
    prompt = torch.randint(0, cfg.vocab_size, (40,), generator=torch.Generator().manual_seed(5)).tolist()

    def run(world_, rank_, group):
        w = synthetic_device_weights(cfg, rank_, world_, seed=9, device=dev, norm_noise=True)
        kv = KVPool(cfg, w.layout.local_kv_heads, 16, 16, dev)
        r = LlamaRunner(w, ecfg, kv, dev, group=group, max_tokens=256)
        r.keep_logits = True
        T = len(prompt)
        bt = torch.zeros(1, 8, dtype=torch.int32, device=dev)
        bt[0, :3] = torch.tensor([1, 2, 3])
        pos = torch.arange(T, device=dev)
        m = StepMeta(ids=torch.tensor(prompt, dtype=torch.int32, device=dev), pos=pos.int(),
                     slot=(bt[0, pos // 16].long() * 16 + pos % 16), block_tables=bt,
                     seq_lens=torch.tensor([T], dtype=torch.int32, device=dev),
                     cu_q=torch.tensor([0, T], dtype=torch.int32, device=dev),
                     last_idx=torch.tensor([T - 1], device=dev), max_q_len=T, decode=False)
        ids = r.forward(m)
        torch.cuda.synchronize()
        return r.last_logits[0].float(), int(ids[0]), w

    full, id1, _ = run(1, 0, None)
    part, id2, w2 = run(world, rank, dist.group.WORLD)
    parts = [torch.empty(n, device=dev) for n in
             [__import__("mesh_b200.models.sharding", fromlist=["x"]).even_split(cfg.vocab_size, world, r)[1]
              for r in range(world)]]
    dist.all_gather(parts, part.contiguous())
    tp = torch.cat(parts)
    err = ((tp - full).norm() / full.norm()).item()
    assert err < 3e-2, err
    assert id2 == int(tp.argmax())


@pytest.fixture(autouse=True)
def _need_gpus():
    if torch.cuda.device_count() < NEED:
        pytest.skip(f"needs {NEED} GPUs")


def test_fused_allreduce_norm_2gpu():
    _run(_ar_check, 2)


def test_fused_allreduce_norm_nvls_2gpu():
    _run(_ar_check, 2, True)


def test_fused_gemm_reduce_scatter_push_2gpu():
    _run(_push_check, 2)


def test_allreduce_bounded_wait_reports_timeout_2gpu():
    _run(_timeout_check, 2)


def test_tp2_logits_match_tp1():
    _run(_tp_logits, 2)
