"""Headline benchmark: decode tokens/s and p50 TTFT of the Llama-3-8B-shaped decoder, tensor
parallel over N B200s of one node (the headline serving configuration: 64 concurrent sessions,
512-token uniform-random prompts, 128 greedy decode tokens, 16-token KV pages, continuous batching).

One bench "step" = one serving episode: submit 64 prompts, prefill them (chunked), decode 128
tokens per session, read the generated tokens back to the host. Timing: CUDA events on the
launching stream, W untimed warm-up episodes, then K timed episodes bracketed by a barrier and
torch.cuda.synchronize(); every time is the MAX over ranks. Weights are N(0, 0.02) random-init
of the named architecture; prompts are synthetic.

    python bench.py [--gpus N --steps K --warmup W]        # N>1: launch under torch.distributed.run
    python bench.py --impl reference                       # the reference arm
    python bench.py --impl torch                           # plain PyTorch arm (cuBLAS + SDPA + NCCL)

``--impl torch`` runs the same engine, episode and timing with ``baselines.torch_tp.TorchTPRunner``
in place of the sm_100a runner: the comparison arm built from library code only.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import torch

BASELINE_METRIC = "decode tokens/s + p50 TTFT, Llama-3 8B/70B TP at 1/2/4/8 B200, max over ranks"
# The reference publishes no throughput figure. The comparison number per GPU count is the plain
# PyTorch arm (``--impl torch``: cuBLAS linears, SDPA over gathered pages, NCCL all-reduce) measured
# with this script on the same B200 pool; None where it has not been measured.
BASELINE_VALUE = {1: 4052.9, 2: 5900.8, 4: 7732.2}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="mesh", choices=["mesh", "reference", "nccl", "torch"])
    ap.add_argument("--model", default="llama3-8b")
    ap.add_argument("--sessions", type=int, default=64)
    ap.add_argument("--prompt-len", type=int, default=512)
    ap.add_argument("--gen", type=int, default=128)
    ap.add_argument("--prefill-chunk", type=int, default=4096)
    ap.add_argument("--layers", type=int, default=0, help="debug only: override layer count (invalid for the metric)")
    ap.add_argument("--no-graphs", action="store_true")
    ap.add_argument("--no-nvls", action="store_true",
                    help="keep the fused all-reduce on plain peer loads (no NVSwitch multimem) at every TP degree")
    ap.add_argument("--prefill-overlap", action="store_true",
                    help="TP prefill: two halves of each chunk on two streams (all-reduce of one overlaps GEMMs of the other)")
    ap.add_argument("--ar-impl", default="auto",
                    choices=["auto", "unfused", "gemm_ar", "oneshot", "twoshot", "push", "push_oneshot", "nccl"],
                    help="TP all-reduce: auto/unfused (separate peer-memory kernel fused with residual + RMSNorm), "
                         "gemm_ar (decode: inside the o_proj/down GEMM launch), pull one/two-shot, "
                         "GEMM->reduce-scatter push, or NCCL")
    return ap.parse_args()


def reference_arm(args):
    line = {"impl": "reference", "unavailable":
            "the reference (saint0x/mesh) is a Rust/Cargo workspace (candle + cudarc); there is no Rust "
            "toolchain or crates.io here and it has no pip-installable package, so it cannot be built or run"}
    print(json.dumps(line), flush=True)


class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons while the timed region runs."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-i", str(self.gpu), "-lms", "200"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        sm.sort()
        med = sm[len(sm) // 2] if sm else None
        return {"sm_mhz": med, "sm_max_mhz": mx or None, "reasons": sorted(reasons), "samples": len(sm)}


def main():
    args = parse()
    if args.impl == "reference":
        reference_arm(args)
        return
    import torch.distributed as dist
    from mesh_b200 import ops
    from mesh_b200.config import EngineConfig, get_preset
    from mesh_b200.engine.serving import Engine
    from mesh_b200.models.llama import KVPool, LlamaRunner
    from mesh_b200.models.weights import synthetic_device_weights
    from mesh_b200.parallel import dist as mdist

    di = mdist.init(timeout_s=120.0)
    world, rank, dev = di.world, di.rank, di.device
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch with torch.distributed.run")
    cfg = get_preset(args.model)
    if args.layers:
        cfg = cfg.replace(num_layers=args.layers)
    S, P, G = args.sessions, args.prompt_len, args.gen
    max_seq = (P + G + 15) // 16 * 16
    ecfg = EngineConfig(tp=world, max_seq_len=max_seq, prefill_chunk_tokens=args.prefill_chunk,
                        use_cuda_graphs=not args.no_graphs, max_decode_batch_size=S,
                        allreduce_impl="nccl" if args.impl == "nccl" else args.ar_impl, nvls=not args.no_nvls,
                        prefill_overlap=args.prefill_overlap or EngineConfig().prefill_overlap)
    w = synthetic_device_weights(cfg, rank, world, seed=1234, device=dev)
    pages = S * (max_seq // 16) + 64
    kv = KVPool(cfg, w.layout.local_kv_heads, pages, 16, dev)
    grp = dist.group.WORLD if world > 1 else None
    if args.impl == "torch":
        from mesh_b200.baselines.torch_tp import TorchTPRunner
        runner = TorchTPRunner(w, ecfg, kv, dev, group=grp, max_tokens=max(args.prefill_chunk + P, S))
    else:
        runner = LlamaRunner(w, ecfg, kv, dev, group=grp, max_tokens=max(args.prefill_chunk + P, S))
    eng = Engine(runner, ecfg, max_batch=S)
    g = torch.Generator().manual_seed(4321)
    prompts_host = torch.randint(0, cfg.vocab_size, (S, P), generator=g, dtype=torch.int32).pin_memory()
    prompts = prompts_host.tolist()

    def episode():
        ev0 = torch.cuda.Event(enable_timing=True)
        ev_p = torch.cuda.Event(enable_timing=True)
        ev_d = torch.cuda.Event(enable_timing=True)
        ev0.record()
        sids = [eng.submit(p, G) for p in prompts]
        while eng.waiting:
            eng.prefill_step()
        ev_p.record()
        while eng.has_work():
            eng.decode_step()
        ev_d.record()
        eng.flush_history()   # device -> host read of the generated tokens
        ev_end = torch.cuda.Event(enable_timing=True)
        ev_end.record()
        torch.cuda.synchronize()
        ttft = sorted(ev0.elapsed_time(eng.sessions[s].ttft_event) for s in sids)
        out = [eng.sessions[s].generated for s in sids]
        assert all(len(o) == G for o in out), "every session must produce its tokens"
        for s in sids:
            del eng.sessions[s]
        return dict(total_ms=ev0.elapsed_time(ev_end), prefill_ms=ev0.elapsed_time(ev_p),
                    decode_ms=ev_p.elapsed_time(ev_d), p50_ttft_ms=ttft[len(ttft) // 2])

    for _ in range(args.warmup):
        episode()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    l0 = ops.LAUNCHES[0]
    res = []
    with ClockSampler(torch.cuda.current_device() if not os.environ.get("CUDA_VISIBLE_DEVICES") else int(
            os.environ["CUDA_VISIBLE_DEVICES"].split(",")[torch.cuda.current_device()])) as clk:
        for _ in range(args.steps):
            res.append(episode())
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
    launches = ops.LAUNCHES[0] - l0
    # diagnostic outside the timed region: device time of one full-batch decode step alone (graph
    # replays back to back, no host work between them), to separate device time from host overhead
    dec_graph_ms = _decode_device_ms(eng, S, dist if world > 1 else None)
    keys = ["total_ms", "prefill_ms", "decode_ms", "p50_ttft_ms"]
    local = torch.tensor([sum(r[k] for r in res) for k in keys[:3]] +
                         [sorted(r["p50_ttft_ms"] for r in res)[len(res) // 2], dec_graph_ms],
                         dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(local, op=dist.ReduceOp.MAX)
    total_ms, prefill_ms, decode_ms, p50_ttft, dec_graph_ms = local.tolist()
    K = args.steps
    decode_tokens = S * (G - 1) * K
    value = decode_tokens / (decode_ms / 1e3)
    e2e = S * G * K / (total_ms / 1e3)
    clocks = clk.summary()
    if rank == 0:
        line = {
            "metric": BASELINE_METRIC, "value": round(value, 1), "unit": "decode tokens/s (aggregate over ranks)",
            "n_gpus": world, "steps": K, "warmup": args.warmup, "ms_per_step": round(total_ms / K, 3),
            "higher_is_better": True, "scaling": "strong",
            "vs_baseline": (round(value / BASELINE_VALUE[world], 3) if BASELINE_VALUE.get(world) else None),
            "dtype": "bf16",
            "data": "synthetic: uniform-random prompt token ids, N(0,0.02) random-init weights",
            "impl": args.impl,
            "p50_ttft_ms": round(p50_ttft, 3), "prefill_ms_per_step": round(prefill_ms / K, 3),
            "decode_ms_per_step": round(decode_ms / K, 3),
            "decode_step_device_ms": round(dec_graph_ms, 4),
            "prefill_tokens_per_s": round(S * P * K / (prefill_ms / 1e3), 1),
            "config": {"model": args.model + ("" if not args.layers else f"-L{args.layers}-INVALID"),
                       "global_batch": S, "seq_len": P, "gen_tokens": G, "kv_page_tokens": 16,
                       "parallelism": f"tp{world}", "prefill_chunk_tokens": args.prefill_chunk,
                       "cuda_graphs": not args.no_graphs, "allreduce": "nccl" if args.impl in ("nccl", "torch") else args.ar_impl,
                       "prefill_overlap": bool(getattr(runner, "overlap_prefill", False)),
                       "nvls": (not args.no_nvls) and world >= 8 and args.impl == "mesh",
                       "l2": "inputs larger than L2 (weights %.1f GB per rank re-read every step)" % (w.nbytes() / 1e9)},
            "e2e": {"value": round(e2e, 1), "unit": "generated tokens/s through Engine.submit/run incl. prefill, "
                    "prompt H2D and token D2H", "h2d_bytes_per_step": S * P * 4 + S * 8 * 3,
                    "d2h_bytes_per_step": S * G * 4},
            "gpu_launches": launches,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    eng.close()
    torch.cuda.synchronize()
    mdist.shutdown()


def _decode_device_ms(eng, batch, dist, reps=20):
    """Mean device time of one decode step at ``batch`` sessions with nothing between steps."""
    d = eng.dec
    b = d.bucket_for(batch)
    for _ in range(3):
        d.step(b)
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(reps):
        d.step(b)
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / reps


if __name__ == "__main__":
    main()
